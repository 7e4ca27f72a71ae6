/*
 * rfsn_b200.h — C ABI of the B200-native RFSN compressed-KV decode path.
 *
 * The reference (dawsonblock/apple, RFSN v10.2) is pure Python on Apple MLX and
 * has no FFI: its boundary is the Python class API (RFSNv10KVCacheMLX,
 * HybridQuantizerMLX, RFSNHybridAttentionMLX, AsyncHierarchicalRouterMLX).
 * Each entry point below replaces the MLX computation behind one of those
 * methods; the comment on each names the reference lines (file:line, relative
 * to the reference project root) whose behaviour it reproduces.
 *
 * Conventions
 *   - Plain C: pointers, sizes, plain structs.  No C++ or torch types.
 *   - Every device pointer is caller-owned; nothing is allocated inside the
 *     library except CUDA's own launch resources.
 *   - Every call is stream-ordered on the given cudaStream_t (passed as void*;
 *     NULL = legacy default stream) and returns an int status (0 = RFSN_OK,
 *     negative = error, see rfsn_status).  No exception crosses the ABI.
 *   - fp16 tensors are passed as uint16_t* holding IEEE binary16 bits.
 *   - A "row" is one (batch, kv-head) pair: row = b * num_kv_heads + h.
 */
#ifndef RFSN_B200_H
#define RFSN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RFSN_ABI_VERSION 1
#define RFSN_MAX_SEGMENTS 256   /* segments per attention call (hot/warm/cold pieces) */
#define RFSN_MAX_ROWS_PER_KV 8  /* query rows (queries x GQA group) sharing one KV head */

typedef enum rfsn_status {
  RFSN_OK = 0,
  RFSN_ERR_INVALID_ARGUMENT = -1,
  RFSN_ERR_UNSUPPORTED = -2,
  RFSN_ERR_CUDA = -3,
  RFSN_ERR_WORKSPACE_TOO_SMALL = -4,
  RFSN_ERR_DEVICE_TIMEOUT = -5, /* a bounded device-side wait expired; outputs are invalid */
  RFSN_ERR_ALIGNMENT = -6
} rfsn_status;

/* Library version (RFSN_ABI_VERSION * 1000 + minor). */
int rfsn_version(void);

/* Human-readable text for a status code (static string). */
const char* rfsn_status_string(int status);

/* Last CUDA error text recorded by a call on this host thread ("" if none). */
const char* rfsn_last_cuda_error(void);

/* ------------------------------------------------------------------------ */
/* Quantizer: the codebooks of HybridQuantizerMLX (quantization.py:296-319).  */
/* ------------------------------------------------------------------------ */
typedef struct rfsn_quantizer {
  const uint16_t* pq_codebooks;  /* fp16 [M][K][ds]  (ProductQuantizerMLX.codebooks, quantization.py:109-115) */
  const uint16_t* rvq_codebooks; /* fp16 [L][Kr][D]  (ResidualVQMLX.codebooks, quantization.py:189-197); NULL if L == 0 */
  int32_t head_dim;              /* D = M * ds (storage.py:53-59) */
  int32_t num_subspaces;         /* M */
  int32_t subspace_dim;          /* ds */
  int32_t pq_codebook_size;      /* K <= 256 (codes are uint8) */
  int32_t rvq_layers;            /* L (0 = PQ only) */
  int32_t rvq_codebook_size;     /* Kr; codes stored as uint8 when Kr <= 256, else uint16 */
  float rvq_threshold;           /* token gets RVQ codes iff ||pq residual||_2 > threshold (quantization.py:216-218) */
  int32_t sparse_topk;           /* S: extension, top-S |error| fp16 entries per token (0 = off) */
} rfsn_quantizer;

/* Compressed code store: the device form of a key/value pair of
 * CompressedTensorMLX (storage.py:75-98).
 *
 * Tokens are grouped in blocks of RFSN_BLOCK_TOKENS (16) consecutive tokens of
 * one row; a block holds every field of the K codes and then of the V codes:
 *
 *   K pq     uint8  [16][M]
 *   K rvq    uint8  [16][L] (Kr <= 256) or uint16 [16][L]   (absent if L == 0)
 *   K active uint8  [16]   1 = RVQ codes apply              (absent if L == 0)
 *   K sp_idx uint8  [16][S]                                  (absent if S == 0)
 *   K sp_val fp16   [16][S]                                  (absent if S == 0)
 *   V ... the same five fields
 *
 * Every sub-array is a multiple of 16 bytes, so blocks and fields stay 16-byte
 * aligned; rfsn_code_block_bytes() gives the block size.  Block b of row r of
 * slot s starts at data + ((s * rows + r) * (cap / 16) + b) * block_bytes, so
 * a run of tokens of one row is one contiguous byte range (one bulk copy).
 * RVQ codes are stored for every token (zero when inactive) next to the
 * activity byte, instead of the reference's (codes, offsets) pair;
 * rvq[active] and flatnonzero(active) give the reference form back. */
#define RFSN_BLOCK_TOKENS 16

typedef struct rfsn_code_store {
  uint8_t* data;     /* [slots][rows][cap / 16][block_bytes] */
  int64_t cap;       /* tokens per row; multiple of 16 */
  int64_t rows;      /* rows per slot (batch * kv heads) */
  int64_t slots;     /* number of slots (1 for a warm store; >1 for a cold chunk pool) */
} rfsn_code_store;

/* Bytes of one 16-token block for this quantizer (K and V fields). */
int64_t rfsn_code_block_bytes(const rfsn_quantizer* qz);

/* Dense fp16 store for exact (hot) tokens: [rows][cap][D]. */
typedef struct rfsn_dense_store {
  const uint16_t* k;
  const uint16_t* v;
  int64_t cap;   /* tokens per row */
  int64_t rows;  /* rows in the store (>= batch * kv heads) */
} rfsn_dense_store;

/* Spill encoder — HybridQuantizerMLX.encode (quantization.py:305-308) =
 * ProductQuantizerMLX.quantize (:124-144) + ResidualVQMLX.encode (:206-252),
 * plus the top-S sparse residual extension; applied per token like
 * _compress_tensor_sequence (:330-343) and written straight into a code store
 * the way RFSNv10KVCacheMLX._add_to_warm / _add_to_cold append (cache.py:122-191).
 *
 * x: fp16, vector (b, t, h) at x[b*stride_b + t*stride_t + h*stride_h], D contiguous.
 * Vector (b, t, h) is written to the K (kv = 0) or V (kv = 1) fields of row b*heads + h,
 * token dst_first + t of slot dst_slot.
 * residual_out (optional, may be NULL): fp16 PQ residual in the same layout as x. */
int rfsn_encode(const rfsn_quantizer* qz, const uint16_t* x, int64_t batch, int64_t tokens, int64_t heads,
                int64_t stride_b, int64_t stride_t, int64_t stride_h, const rfsn_code_store* dst, int32_t kv,
                int64_t dst_slot, int64_t dst_first, uint16_t* residual_out, void* stream);

/* K and V of the same tokens in one launch: rfsn_encode(k, kv = 0) and rfsn_encode(v, kv = 1)
 * with the same shape, strides and destination, no residual output.  The reference encodes
 * them with two _compress_tensor_sequence calls (_add_to_warm, cache.py:122-132); at decode a
 * step appends one token per row, and one launch instead of two halves the encoder's fixed
 * cost.  Same codes as the two calls. */
int rfsn_encode_kv(const rfsn_quantizer* qz, const uint16_t* k, const uint16_t* v, int64_t batch, int64_t tokens,
                   int64_t heads, int64_t stride_b, int64_t stride_t, int64_t stride_h, const rfsn_code_store* dst,
                   int64_t dst_slot, int64_t dst_first, void* stream);

/* Decode compressed tokens to dense fp16 — _decode_compressed_tensor (quantization.py:394-402),
 * i.e. fp16(pq_decode + rvq_correction) (:319) plus the sparse residual added in fp32 and
 * rounded once.  K (kv = 0) or V (kv = 1) tokens [first, first+count) of every row of slot `slot`; token i of row
 * (b, h) goes to out[b*stride_b + i*stride_t + h*stride_h] (D contiguous).  This is what
 * RFSNv10KVCacheMLX.materialize_window (cache.py:344-393) returns for warm/cold tokens. */
int rfsn_decode_codes(const rfsn_quantizer* qz, const rfsn_code_store* src, int32_t kv, int64_t slot,
                      int64_t first, int64_t count, int64_t batch, int64_t heads, uint16_t* out, int64_t stride_b,
                      int64_t stride_t, int64_t stride_h, void* stream);

/* One contiguous run of window tokens in one store. */
typedef struct rfsn_segment {
  int32_t store;   /* 0 = hot dense store, 1 = warm code store, 2 = cold code pool */
  int32_t slot;    /* slot in the store (cold pool) */
  int32_t first;   /* first token index inside the row storage */
  int32_t count;   /* number of tokens */
  int32_t pos0;    /* global sequence position of token `first` (causal masking) */
  int32_t reserved[3];
} rfsn_segment;

/* Output all-gather fused into decode attention, over NVLink peer memory.
 *
 * Work is sharded across the GPUs of one node by sequence (rank r holds sequences
 * [seq_offset, seq_offset + batch) of total_seqs); the output projection needs every
 * sequence's attention output on every rank.  Instead of a separate all-gather, the CTA that
 * merges a row stores its fp16 output straight into every rank's gathered-output buffer (plain
 * peer stores through IPC-mapped addresses), and the launch's last CTA then signals every rank
 * and waits (bounded, 1 s) until every rank has signalled the same launch, after which it copies
 * the complete gathered output into out_full.
 *
 * buffers[k]: rank k's gathered-output buffers, 2 x total_seqs x queries x q_heads x head_dim fp16
 * (two, used by launch parity, so a rank one launch ahead never overwrites a buffer another rank
 * is still copying); flags[k]: rank k's num_ranks uint64 flag words; step: this rank's uint64
 * launch counter.  All of buffers[rank], flags[rank] and step live in one allocation made by
 * rfsn_peer_alloc (zeroed); the other ranks' come from rfsn_peer_open.  Every rank must make the
 * same sequence of gathered launches.  Ranks must be on distinct GPUs: the wait is on other
 * GPUs' launches. */
#define RFSN_MAX_PEERS 8
typedef struct rfsn_peer_gather {
  int32_t num_ranks;
  int32_t rank;
  int64_t seq_offset;
  int64_t total_seqs;
  uint16_t* buffers[RFSN_MAX_PEERS];
  uint64_t* flags[RFSN_MAX_PEERS];
  uint64_t* step;
  uint16_t* out_full;  /* [total_seqs][queries][q_heads][head_dim] fp16 on this device */
} rfsn_peer_gather;

/* Peer-visible device memory for rfsn_peer_gather: cudaMalloc of `bytes` (zeroed) and its CUDA
 * IPC handle (64 bytes written to ipc_handle); rfsn_peer_open maps another process's allocation
 * from its handle on the current device; rfsn_peer_close unmaps it; rfsn_peer_free frees one's
 * own allocation. */
int rfsn_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int rfsn_peer_open(const void* ipc_handle, void** ptr);
int rfsn_peer_close(void* ptr);
int rfsn_peer_free(void* ptr);

/* Fused decode attention — RFSNv10KVCacheMLX.attention_forward (cache.py:395-428) =
 * materialize_window (:344-393) + _blockwise_exact_attention (attention.py:39-105),
 * without materialising the window: PQ/RVQ/sparse codes are decoded inside a
 * flash-decoding split-K kernel and partial (max, sum, acc) triples are merged by
 * log-sum-exp.  Also covers RFSNHybridAttentionMLX.__call__ (attention.py:150-170).
 *
 * q / out: fp16 [batch][queries][q_heads][D]; query head hq reads KV head hq / (q_heads/kv_heads).
 *       out may be device memory or pinned (mapped) host memory, which the kernel then writes
 *       over the bus: the caller synchronizes the stream before reading it.
 * qpos: int32 [batch][queries][q_heads] global positions; key at position p is visible
 *       iff p <= qpos (causal); ignored when causal == 0.
 * segments: host array in window (position) order; their token counts sum to the window.
 * An empty window writes zeros (cache.py:417-418). */
typedef struct rfsn_attn_args {
  const uint16_t* q;
  const int32_t* qpos;
  uint16_t* out;
  int32_t batch, queries, q_heads, kv_heads, head_dim;
  int32_t causal;
  float scale;                     /* head_dim ** -0.5 in the reference (cache.py:424) */
  rfsn_dense_store hot;
  rfsn_code_store warm;
  rfsn_code_store cold;
  const rfsn_segment* segments;
  int32_t num_segments;
  int32_t num_ctas;                /* 0 = one CTA per SM */
  void* workspace;                 /* device scratch, >= rfsn_attention_workspace_size() bytes.  Its first
                                      bytes hold a launch counter and per-row completion tickets that every
                                      launch advances (so CUDA-graph replays of one call stay correct):
                                      it must be zeroed once when allocated; reuse it without clearing.
                                      Calls that overlap in time must not share a workspace. */
  size_t workspace_bytes;
  int32_t* device_status;          /* optional device int32, set non-zero on a device-side failure: 1/2 a bounded
                                      wait timed out, 4 a row ticket could not be taken */
  int64_t q_batch_stride;          /* elements from one sequence's queries to the next (a multiple of 8, at least
                                      queries*q_heads*head_dim); 0 = packed.  Lets q be a view of a wider
                                      projection output. */
  const rfsn_peer_gather* gather;  /* optional fused output all-gather over peer memory (NULL = none);
                                      device_status 5 = a peer's signal did not arrive in time */
} rfsn_attn_args;

/* Bytes of device workspace rfsn_decode_attention needs for these arguments. */
int rfsn_attention_workspace_size(const rfsn_attn_args* args, const rfsn_quantizer* qz, size_t* bytes);

int rfsn_decode_attention(const rfsn_attn_args* args, const rfsn_quantizer* qz, void* stream);

/* rfsn_decode_attention with the query in HOST memory (the reference-facing call with host
 * buffers).  q_host: the packed fp16 query [batch][queries][q_heads][D] (pinned memory lets the
 * copy run asynchronously); q_stage: a device buffer of the same size the call copies it into on
 * the stream (args->q is ignored; args->q_batch_stride must be 0 or the packed stride).  args->out
 * may be device memory or pinned (mapped) host memory.  synchronize != 0: return after the stream
 * has finished, so a host out holds the result.  Replaces the upload + attention_forward + read of
 * cache.py:395-428 driven from a host caller. */
int rfsn_decode_attention_host(const rfsn_attn_args* args, const rfsn_quantizer* qz, const uint16_t* q_host,
                               uint16_t* q_stage, int synchronize, void* stream);

/* Allocation-free decode attention.  No counterpart in the reference: it is an
 * addition for callers that cannot allocate device memory when they run
 * attention (a host binding that holds only q/out/store pointers, a runtime
 * whose memory is fixed up front).  Same arguments and results as
 * rfsn_decode_attention, except that args->workspace / workspace_bytes are
 * ignored: partials go to a fixed 4 MiB buffer per device inside the library
 * (RFSN_NOALLOC_SCRATCH_BYTES).  Returns RFSN_ERR_WORKSPACE_TOO_SMALL when the
 * call needs more than that (rfsn_attention_workspace_size reports the need).
 * The first call on each device looks the buffer up and may load the module:
 * make it before capturing the stream.  Calls that overlap in time on one
 * device share the buffer and race; calls ordered on one stream are safe. */
#define RFSN_NOALLOC_SCRATCH_BYTES (4u << 20)
int rfsn_decode_attention_noalloc(const rfsn_attn_args* args, const rfsn_quantizer* qz, void* stream);

/* Centroid routing of the cold tier (extension; the reference's router, storage.py:166-182,
 * orders chunks by distance from the position and the cache then decodes every chunk the window
 * overlaps, cache.py:293-342).  centroids: fp32 [num_chunks][batch * kv_heads][head_dim], the
 * mean decoded key of each chunk per row.  q: fp16 [batch][queries][q_heads][head_dim] with
 * batch stride q_batch_stride elements (0 = packed).  scores[c] = max over (b, i, h) of
 * q[b, i, h] . centroids[c][b * kv_heads + h / (q_heads / kv_heads)] (fp32); ids[0..k) = the k
 * highest-scoring chunk indices, descending, ties to the lower index.  scratch: num_chunks bytes
 * of device memory.  k <= 64.  Device outputs, stream-ordered. */
int rfsn_route_topk(const uint16_t* q, int64_t q_batch_stride, int32_t batch, int32_t queries, int32_t q_heads,
                    int32_t kv_heads, int32_t head_dim, const float* centroids, int32_t num_chunks, int32_t k,
                    float* scores, int32_t* ids, uint8_t* scratch, void* stream);

/* Cold tier transfer — replaces load_compressed_chunk / np.load in the router's
 * executor (storage.py:138-140, 226-234): one cudaMemcpyAsync of `bytes` from
 * pinned host memory to device memory on `stream` (the router's side stream),
 * followed by a record of `event` (a cudaEvent_t, may be NULL) on that stream. */
int rfsn_cold_prefetch(void* dst_device, const void* src_pinned_host, size_t bytes, void* stream, void* event);

/* Device-to-host counterpart used when warm chunks age out to the cold tier
 * (save_compressed_chunk, storage.py:117-135). */
int rfsn_cold_evict(void* dst_pinned_host, const void* src_device, size_t bytes, void* stream);

/* Decoder-layer element-wise steps, one launch each (RFSNDecoderLayerMLX,
 * rfsn_v10_mlx_ane_complete.py:114-172, which evaluates them as chains of
 * tensor operations).
 *
 * rfsn_rmsnorm_f16: y[r] = fp16((x[r] * rsqrt(mean(x[r]^2) + eps)) * weight) in
 * fp32, for `rows` contiguous fp16 rows of `dim` features and an fp32 weight of
 * `dim` (the layer's RMSNorm / mlx.nn.RMSNorm).
 *
 * rfsn_gelu_tanh_f16: y = 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))) over
 * n fp16 values, rounded to fp16 after every operation as the layer's fp16
 * expression is (attention.py:137-138).  x and y may alias. */
int rfsn_rmsnorm_f16(const uint16_t* x, const float* weight, uint16_t* y, int64_t rows, int dim, float eps,
                     void* stream);
int rfsn_gelu_tanh_f16(const uint16_t* x, uint16_t* y, int64_t n, void* stream);

/* sum = fp16(x + b) (one rounding of the fp32 sum, as the layer's fp16 residual add) and
 * y = rfsn_rmsnorm_f16(sum) in one launch: the layer's `hidden = residual + attn_out`
 * followed by its FFN RMSNorm (RFSNDecoderLayerMLX.__call__, rfsn_v10_mlx_ane_complete.py:114-172). */
int rfsn_add_rmsnorm_f16(const uint16_t* x, const uint16_t* b, uint16_t* sum, const float* weight, uint16_t* y,
                         int64_t rows, int dim, float eps, void* stream);

/* Weight-streaming projection for decode-sized row counts: y[M][N] = x[M][K] W[N][K]^T with fp32
 * accumulation, fp16 result — the decoder layers' projections (mlx.nn.Linear in RFSNDecoderLayerMLX,
 * rfsn_v10_mlx_ane_complete.py:114-172; _linear, llama32_adapter.py:492-494), with an optional fused
 * epilogue: 0 none, 1 y = fp16(fp16(acc) + r) (the residual add after o_proj / ffn_down), 2 y =
 * gelu_tanh(fp16(acc)) rounded to fp16 after every operation (the FFN activation, attention.py:
 * 137-138).  M <= 32, N % 64 == 0, K % 128 == 0; row strides in elements, x and W rows 16-byte
 * aligned.  The workspace (rfsn_linear_workspace_size bytes, 256-byte aligned) holds per-tile
 * tickets, which every completed launch leaves at zero, and fp32 partials: zero it once when
 * allocated (and again after a launch that set a device status), reuse it without clearing,
 * never share it between calls that overlap in time (consecutive calls on one stream, of any
 * shapes, may share it).  The kernel is launched as a programmatic dependent launch: it may begin
 * streaming W while the previous kernel on the stream finishes, and reads x, r, the workspace
 * and writes y only after that kernel has completed. */
int rfsn_linear_workspace_size(int M, int N, int K, size_t* bytes);
int rfsn_linear_f16(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t ldw, const uint16_t* r, int64_t ldr,
                    uint16_t* y, int64_t ldy, int M, int N, int K, int epilogue, void* workspace,
                    size_t workspace_bytes, int32_t* device_status, void* stream);

/* Affine low-bit codebook quantization — the reference's quantize_codebooks_for_ane path
 * (_quantize_matrix / _dequantize_matrix, quantization.py:36-89, used at :159-175 and :277-293),
 * which calls MLX's mx.quantize / mx.dequantize (affine mode).  For each group of `group`
 * consecutive elements of a row of w (fp32 [rows][cols], cols % group == 0, group <= 128):
 * scale = (max - min) / (2^bits - 1), bias = min, q = clip(round_half_even((w - bias) / scale),
 * 0, 2^bits - 1) and dequantized = q * scale + bias, all fp32 (a constant group: scale 0, q 0).
 * Outputs: q uint8 [rows][cols], scales and biases fp32 [rows][cols / group], dequantized fp32
 * [rows][cols]. */
int rfsn_affine_quantize_f32(const float* w, int64_t rows, int cols, int group, int bits, uint8_t* q, float* scales,
                             float* biases, float* dequantized, void* stream);

/* Llama adapter layer element-wise steps (Llama32DecoderLayerMLX, llama32_adapter.py:417-662), one
 * launch each, in the adapter's operation order and rounding points:
 *
 * rfsn_llama_rmsnorm_f16: y[r] = fp16(x[r] / sqrt(mean(x[r]^2) + eps) * weight) in fp32 with an fp16
 * weight (_rms_norm, :497-500).  With b != NULL the row is first sum = fp16(x + b) (the residual
 * add before the post-attention norm) and sum is normalised.
 *
 * rfsn_rope_f16: y = fp16(x * cos + rotate_half(x) * sin) in fp32 (_apply_rope, :555-568) for
 * x [batch][seq][heads][dim] (element strides; dim contiguous) and fp16 tables [seq][dim]; y may
 * alias x.
 *
 * rfsn_silu_mul_f16: y = fp16(fp16(g * sigmoid(g)) * up) over n values (_silu and the gated
 * product of _forward_mlp, :502-504, 584-589). */
int rfsn_llama_rmsnorm_f16(const uint16_t* x, const uint16_t* b, uint16_t* sum, const uint16_t* weight, uint16_t* y,
                           int64_t rows, int dim, float eps, void* stream);
int rfsn_rope_f16(const uint16_t* x, int64_t stride_b, int64_t stride_s, int64_t stride_h, uint16_t* y,
                  int64_t y_stride_b, int64_t y_stride_s, int64_t y_stride_h, const uint16_t* cos_table,
                  const uint16_t* sin_table, int64_t batch, int seq, int heads, int dim, void* stream);
int rfsn_silu_mul_f16(const uint16_t* gate, const uint16_t* up, uint16_t* y, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RFSN_B200_H */
