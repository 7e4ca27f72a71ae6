// linear.cu — weight-streaming projection for decode-sized row counts.
//
// The decoder layers' projections (RFSNDecoderLayerMLX, rfsn_v10_mlx_ane_complete.py:
// 114-172; the Llama adapter's _linear, llama32_adapter.py:492-494) multiply a
// few activation rows (one per sequence at decode: M <= 32) by a weight matrix
// W [N][K] fp16 that is far larger than L2's share of one step, so the product
// is bound by streaming W once from HBM.  y[M][N] = x[M][K] W^T, fp32
// accumulation, fp16 result, with an optional fused epilogue:
//
//   0  y = fp16(acc)
//   1  y = fp16(fp16(acc) + r)            the layer's residual add after ffn_down
//   2  y = gelu_tanh(fp16(acc))           the layer's FFN activation, fp16 after every operation
//
// Work split (stream-K).  W is cut into 64-row tiles and K into 128-wide chunks;
// one work item is one (tile, chunk), items numbered tile-major.  CTA c of G takes
// the contiguous items [c I / G, (c + 1) I / G), so every CTA streams the same
// number of W bytes within one chunk.  A CTA accumulates a tile's chunks in
// registers; a tile it covers whole gets its epilogue straight from registers.
// A tile cut by a range boundary is covered by a few consecutive CTAs: each
// writes its fp32 partial to a workspace slot, and the CTA whose arrival on the
// tile's ticket comes last sums the partials in CTA order (= K order, so the
// result does not depend on timing), applies the epilogue and resets the ticket
// to zero for the next launch.  Tickets are taken once, after the CTA's last
// item, as one acquire-release atomic add per cut tile, so the stream never stops
// for them and the tail costs two round trips to L2.
//
// In a CTA, a producer warp copies each item's W slab (64 rows x 128) and x slab
// (32 rows x 128; rows past M arrive as zeros) into a shared-memory ring with
// 2-D tensor-map copies (cp.async.bulk.tensor, four 64-column boxes per item)
// in the 128-byte swizzled layout, so that 8-row ldmatrix reads fall in distinct
// banks; the mbarriers that guard the stages are waited with bounds.  Eight
// consumer warps run mma.sync m16n8k16: warp w owns activation rows 16 (w / 4)
// .. + 16 and W rows 16 (w % 4) .. + 16 of the tile.
//
// Programmatic dependent launch.  The kernel is launched so that it may start
// while the kernel before it in the stream finishes: the producer issues the W
// copies of its first stages (W does not depend on earlier kernels) and only then
// waits for the earlier grids (griddepcontrol.wait) before copying x; consumers
// wait likewise before they touch global memory.  Each CTA also lets the next
// launch start early (griddepcontrol.launch_dependents).  The ring takes about
// 97 KB, so a CTA of the next launch fits beside one of this launch on an SM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "rfsn_api_internal.h"
#include "rfsn_attn_util.cuh"
#include "rfsn_common.cuh"
#include "rfsn_elementwise.cuh"

namespace rfsn {

constexpr int kLinTile = 64;       // W rows per tile
constexpr int kLinRows = 32;       // activation rows (M <= 32)
constexpr int kLinChunk = 128;     // K per work item
constexpr int kLinBox = 64;        // columns per tensor-map box (128 bytes: the swizzle span)
constexpr int kLinConsumers = 8;   // consumer warps
constexpr int kLinStages = 4;
constexpr int kLinThreads = (kLinConsumers + 1) * 32;
constexpr int kLinPartial = kLinRows * kLinTile;  // fp32 elements of one partial slot
constexpr int kLinWBox = kLinTile * kLinBox * 2;  // bytes of one W box (64 rows x 128 B)
constexpr int kLinXBox = kLinRows * kLinBox * 2;  // bytes of one x box (32 rows x 128 B)
constexpr int kLinXOff = 2 * kLinWBox;            // x boxes follow the two W boxes
constexpr int kLinStageBytes = 2 * kLinWBox + 2 * kLinXBox;  // a multiple of 1024
constexpr int kLinCtl = 256;                                 // barriers and flags ahead of the ring
constexpr int kLinSmem = kLinCtl + 1024 + kLinStages * kLinStageBytes;  // + alignment of the ring to 1024

struct alignas(64) LinParams {
  CUtensorMap wmap;    // W [N][K]: boxes of 64 rows x 64 columns, 128-byte swizzle
  CUtensorMap xmap;    // x [M][K]: boxes of 32 rows x 64 columns (rows past M read as zeros)
  const uint16_t* r;   // epilogue 1: [M][N] fp16, row stride ldr
  uint16_t* y;         // [M][N] fp16, row stride ldy
  int64_t ldr, ldy;
  int M, N, K, splits, epilogue;
  int64_t items;       // tiles * splits
  float* partial;      // [grid][2][32][64] fp32: a CTA's first and last tile
  unsigned* tickets;   // one per tile, zero between launches (the last arrival resets it)
  int32_t* dev_status;
};

// 2-D tensor-map copy of the box at column x, row y into shared memory; completion is
// reported as transaction bytes on `bar` (a CTA outside a cluster is its own cluster).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of 16-byte chunk c of row r in a box stored with the 128-byte swizzle
// (rows of 128 bytes; chunk c of row r sits at chunk c ^ (r % 8)).
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// Bounded barrier of the consumer warps on an mbarrier (one arrive per warp); false when it
// timed out or another thread gave up (abort set), so no warp is left waiting on the others.
__device__ __forceinline__ bool lin_sync(uint64_t* bar, uint32_t& phase, volatile int* abort) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  const bool ok = mbar_wait_bounded(bar, phase, abort);
  phase ^= 1u;
  __syncwarp();
  if (!ok) *abort = 1;
  return ok;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// First item of CTA c: floor(c I / G).  The CTA holding item i: floor(((i + 1) G - 1) / I).
__device__ __forceinline__ int64_t lin_first(int64_t c, int64_t items, int64_t grid) { return c * items / grid; }
__device__ __forceinline__ int64_t lin_owner(int64_t i, int64_t items, int64_t grid) {
  return ((i + 1) * grid - 1) / items;
}

// The epilogue of one output element from its fp32 sum.
__device__ __forceinline__ uint16_t lin_out(const LinParams& p, float s, int m, int64_t n) {
  uint16_t h = f2h(s);
  if (p.epilogue == 1) h = f2h(__fadd_rn(h2f(h), h2f(p.r[(int64_t)m * p.ldr + n])));
  else if (p.epilogue == 2) h = gelu_tanh_f16(h);
  return h;
}

__global__ void __launch_bounds__(kLinThreads, 2) rfsn_linear_kernel(const __grid_constant__ LinParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kLinStages;
  uint64_t* sync_bar = empty + kLinStages;  // bounded barrier of the consumer warps
  volatile int* flags = reinterpret_cast<volatile int*>(sync_bar + 1);  // [0] abort, [1] [2] boundary tiles won
  // the swizzled boxes need 1024-byte aligned destinations
  unsigned char* ring = smem + ((smem_u32(smem) + kLinCtl + 1023u) & ~1023u) - smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t lo = lin_first(blockIdx.x, p.items, G), hi = lin_first(blockIdx.x + 1, p.items, G);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLinStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLinConsumers);
    }
    mbar_init(sync_bar, kLinConsumers);
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch();

  if (warp == kLinConsumers) {  // ===== producer: four tensor-map boxes per item, issued by lane 0 =====
    constexpr uint32_t tx_bytes = kLinStageBytes;  // out-of-range x rows are written too (as zeros)
    const int pre = hi - lo < kLinStages ? (int)(hi - lo) : kLinStages;
    // the W boxes of the first stages go out before waiting for earlier grids (none writes W)
    if (lane == 0) {
      for (int k = 0; k < pre; ++k) {
        const int64_t i = lo + k, tile = i / p.splits, chunk = i - tile * p.splits;
        unsigned char* sb = ring + k * kLinStageBytes;
        mbar_arrive_expect_tx(&full[k], tx_bytes);
        for (int bx = 0; bx < 2; ++bx)
          tma_load_2d(sb + bx * kLinWBox, &p.wmap, (int)(chunk * kLinChunk + bx * kLinBox), (int)(tile * kLinTile),
                      &full[k]);
      }
    }
    griddep_wait();
    if (lane == 0) {
      for (int k = 0; k < pre; ++k) {
        const int64_t chunk = (lo + k) % p.splits;
        unsigned char* sb = ring + k * kLinStageBytes + kLinXOff;
        for (int bx = 0; bx < 2; ++bx)
          tma_load_2d(sb + bx * kLinXBox, &p.xmap, (int)(chunk * kLinChunk + bx * kLinBox), 0, &full[k]);
      }
    }
    int stage = pre % kLinStages;
    uint32_t phase = pre / kLinStages, inflight = (1u << pre) - 1u, inflight_parity = 0;
    bool ok = true;
    for (int64_t i = lo + pre; i < hi; ++i) {
      const int64_t tile = i / p.splits, chunk = i - tile * p.splits;
      int got = 1;
      if (lane == 0 && !mbar_wait_bounded(&empty[stage], phase ^ 1u, flags)) {
        flags[0] = 1;
        if (p.dev_status) atomicExch(p.dev_status, kDevStatusTimeoutEmpty);
        got = 0;
      }
      if (!__shfl_sync(0xffffffffu, got, 0)) {
        ok = false;
        break;
      }
      unsigned char* sb = ring + stage * kLinStageBytes;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[stage], tx_bytes);
        for (int bx = 0; bx < 2; ++bx) {
          const int kx = (int)(chunk * kLinChunk + bx * kLinBox);
          tma_load_2d(sb + bx * kLinWBox, &p.wmap, kx, (int)(tile * kLinTile), &full[stage]);
          tma_load_2d(sb + kLinXOff + bx * kLinXBox, &p.xmap, kx, 0, &full[stage]);
        }
      }
      __syncwarp();
      inflight |= 1u << stage;
      inflight_parity = (inflight_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == kLinStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (lane == 0 && !ok) {  // leave no copy writing into the CTA's shared memory
      for (int k = 0; k < kLinStages; ++k) {
        if (!((inflight >> k) & 1u)) continue;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full[k], (inflight_parity >> k) & 1u))
          if (global_timer_ns() - t0 > kWaitLimitNs) break;
      }
    }
    return;
  }

  // ===== consumers: warp w computes activation rows 16 (w / 4) + [0, 16) x W rows 16 (w % 4) + [0, 16) =====
  griddep_wait();  // before any global access: partials, tickets, residual and outputs
  const int mt = warp >> 2, nq = warp & 3;
  const int g = lane >> 2, t4 = lane & 3;
  // ldmatrix rows and 16-byte chunk offsets (0 or 1 within a k16 step) of this lane
  const int a_row = 16 * mt + (lane & 15), a_c = lane >> 4;
  const int b_row = 16 * nq + ((lane >> 4) << 3) + (lane & 7), b_c = (lane >> 3) & 1;
  const int64_t first_tile = lo / p.splits, last_tile = (hi - 1) / p.splits;
  int stage = 0;
  uint32_t phase = 0, sync_phase = 0;
  bool ok = true;
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int64_t i = lo; i < hi; ++i) {
    const int64_t tile = i / p.splits;
    const int chunk = (int)(i - tile * p.splits);
    if (!mbar_wait_bounded(&full[stage], phase, flags)) {
      flags[0] = 1;
      if (p.dev_status) atomicExch(p.dev_status, kDevStatusTimeoutFull);
      ok = false;
      break;
    }
    const unsigned char* sb = ring + stage * kLinStageBytes;
#pragma unroll
    for (int ks = 0; ks < kLinChunk / 16; ++ks) {  // k16 step ks: box ks / 4, chunks 2 (ks % 4) + {0, 1}
      const int bx = ks >> 2, c2 = 2 * (ks & 3);
      uint32_t a[4], b[4];
      ldsm_x4(a, sb + kLinXOff + bx * kLinXBox + swz(a_row, c2 + a_c));
      ldsm_x4(b, sb + bx * kLinWBox + swz(b_row, c2 + b_c));
      mma16816(acc[0], a, b[0], b[1]);
      mma16816(acc[1], a, b[2], b[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);  // the slab is consumed
    if (++stage == kLinStages) {
      stage = 0;
      phase ^= 1u;
    }
    if (chunk != p.splits - 1 && i != hi - 1) continue;
    // the tile (or this CTA's share of it) is complete
    if (tile * p.splits >= lo && chunk == p.splits - 1) {  // whole tile here: epilogue from registers
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int m = 16 * mt + g + 8 * h;
          const int64_t n = tile * kLinTile + 16 * nq + 8 * u + 2 * t4;
          if (m < p.M) {
            p.y[(int64_t)m * p.ldy + n] = lin_out(p, acc[u][2 * h], m, n);
            p.y[(int64_t)m * p.ldy + n + 1] = lin_out(p, acc[u][2 * h + 1], m, n + 1);
          }
        }
    } else {  // a share of a tile cut by the range: slot 0 for the first tile, 1 for the last
      float* part = p.partial + ((size_t)blockIdx.x * 2 + (tile == first_tile ? 0 : 1)) * kLinPartial;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int col = 16 * nq + 8 * u + 2 * t4;
        *reinterpret_cast<float2*>(part + (16 * mt + g) * kLinTile + col) = make_float2(acc[u][0], acc[u][1]);
        *reinterpret_cast<float2*>(part + (16 * mt + g + 8) * kLinTile + col) = make_float2(acc[u][2], acc[u][3]);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
  }

  // tiles cut by this CTA's range: one ticket each; the last arrival sums the shares in CTA order
  const bool cut0 = first_tile * p.splits < lo || hi < (first_tile + 1) * p.splits;
  const bool cut1 = last_tile != first_tile && hi < (last_tile + 1) * p.splits;
  if (ok && (cut0 || cut1)) {
    ok = lin_sync(sync_bar, sync_phase, flags);  // every share of this CTA is written
    if (ok && threadIdx.x < 2) {  // thread b takes the ticket of cut tile b, both in flight together
      const int b = threadIdx.x;
      int won = 0;
      if (b == 0 ? cut0 : cut1) {
        const int64_t t = b == 0 ? first_tile : last_tile;
        const unsigned target = (unsigned)(lin_owner(t * p.splits + p.splits - 1, p.items, G) -
                                           lin_owner(t * p.splits, p.items, G) + 1);
        // release publishes this CTA's share to the arrival that completes the count; acquire
        // makes the other shares visible to it
        const unsigned prev = atom_add_acq_rel_gpu(p.tickets + t, 1u);
        if (prev + 1u == target) {
          won = 1;
          p.tickets[t] = 0u;  // every arrival of this launch is in: ready for the next launch
        } else if (prev + 1u > target && p.dev_status) {
          atomicExch(p.dev_status, kDevStatusTicket);  // the ticket held counts of an unfinished launch
        }
      }
      flags[1 + b] = won;
    }
    if (ok) ok = lin_sync(sync_bar, sync_phase, flags);
    for (int b = 0; ok && b < 2; ++b) {
      if (!flags[1 + b]) continue;
      const int64_t t = b == 0 ? first_tile : last_tile;
      const int64_t c0 = lin_owner(t * p.splits, p.items, G), c1 = lin_owner(t * p.splits + p.splits - 1, p.items, G);
      // every contributor after the first starts its range inside tile t (slot 0); the first holds
      // t as its last tile (slot 1) unless its range starts exactly at the tile's first chunk
      const float4* share0 = reinterpret_cast<const float4*>(
          p.partial + (c0 * 2 + (lin_first(c0, p.items, G) < t * p.splits ? 1 : 0)) * kLinPartial);
      const int n_shares = (int)(c1 - c0 + 1);
      // four columns per thread; up to eight shares in flight before they are summed in order
      for (int i4 = threadIdx.x; i4 < p.M * (kLinTile / 4); i4 += kLinConsumers * 32) {
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k0 = 0; k0 < n_shares; k0 += 8) {
          float4 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (k0 + u < n_shares) {
              const float4* sh = k0 + u == 0 ? share0
                                              : reinterpret_cast<const float4*>(p.partial + (c0 + k0 + u) * 2 * kLinPartial);
              v[u] = __ldcg(sh + i4);
            }
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (k0 + u < n_shares) {
              s[0] = __fadd_rn(s[0], v[u].x); s[1] = __fadd_rn(s[1], v[u].y);
              s[2] = __fadd_rn(s[2], v[u].z); s[3] = __fadd_rn(s[3], v[u].w);
            }
        }
        const int m = i4 / (kLinTile / 4);
        const int64_t n0 = t * kLinTile + 4 * (i4 - m * (kLinTile / 4));
#pragma unroll
        for (int e = 0; e < 4; ++e) p.y[(int64_t)m * p.ldy + n0 + e] = lin_out(p, s[e], m, n0 + e);
      }
    }
  }
}

}  // namespace rfsn

namespace rfsn {

struct LinPlan {
  LinParams p;
  int grid;
  size_t ws_bytes;
  int64_t ctl_bytes;  // bytes of the partial slots; the tickets follow
};

static int lin_plan(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t ldw, const uint16_t* r, int64_t ldr,
                    uint16_t* y, int64_t ldy, int M, int N, int K, int epilogue, LinPlan& pl) {
  if (M <= 0 || M > kLinRows || N <= 0 || K <= 0 || epilogue < 0 || epilogue > 2) return RFSN_ERR_INVALID_ARGUMENT;
  if (N % kLinTile || K % kLinChunk) return RFSN_ERR_UNSUPPORTED;
  if (!x || !w || !y || (epilogue == 1 && !r)) return RFSN_ERR_INVALID_ARGUMENT;
  if (ldx < K || ldw < K || ldy < N || (epilogue == 1 && ldr < N)) return RFSN_ERR_INVALID_ARGUMENT;
  // every bulk copy starts on a 16-byte boundary: row strides and bases multiples of 16 bytes
  if ((ldx % 8) || (ldw % 8) || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return RFSN_ERR_ALIGNMENT;
  LinParams& p = pl.p;
  p = LinParams{};
  p.r = r; p.y = y;
  p.ldr = ldr; p.ldy = ldy;
  p.M = M; p.N = N; p.K = K; p.splits = K / kLinChunk; p.epilogue = epilogue;
  const int64_t tiles = N / kLinTile;
  p.items = tiles * p.splits;
  if (p.items >= (int64_t)1 << 40) return RFSN_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  pl.grid = (int)(p.items < sms ? p.items : sms);
  // one layout for every shape, so calls of different shapes can share a workspace: the partial
  // slots of one CTA per SM first, then the tickets (a call leaves the tickets it does not use
  // untouched, and every ticket it uses back at zero)
  pl.ctl_bytes = (int64_t)sms * 2 * kLinPartial * sizeof(float);
  pl.ws_bytes = (size_t)pl.ctl_bytes + (size_t)align_up(tiles * 4, 256);
  return RFSN_OK;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
static PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// A [rows][cols] fp16 matrix with row stride ld (elements) as boxes of box_rows x 64 columns,
// stored with the 128-byte swizzle; boxes past the last row read zeros.
static int encode_matrix(CUtensorMap* map, const uint16_t* base, int64_t rows, int64_t cols, int64_t ld,
                         int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_tiled();
  if (!fn) return RFSN_ERR_CUDA;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kLinBox, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RFSN_OK : RFSN_ERR_INVALID_ARGUMENT;
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_linear_workspace_size(int M, int N, int K, size_t* bytes) {
  if (!bytes) return RFSN_ERR_INVALID_ARGUMENT;
  static const uint16_t dummy[8] __attribute__((aligned(16))) = {0};
  LinPlan pl;
  const int st = lin_plan(dummy, K, dummy, K, nullptr, N, const_cast<uint16_t*>(dummy), N, M, N, K, 0, pl);
  if (st != RFSN_OK) return st;
  *bytes = pl.ws_bytes;
  return RFSN_OK;
}

extern "C" int rfsn_linear_f16(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t ldw, const uint16_t* r,
                               int64_t ldr, uint16_t* y, int64_t ldy, int M, int N, int K, int epilogue,
                               void* workspace, size_t workspace_bytes, int32_t* device_status, void* stream) {
  LinPlan pl;
  int st = lin_plan(x, ldx, w, ldw, r, ldr, y, ldy, M, N, K, epilogue, pl);
  if (st != RFSN_OK) return st;
  if (!workspace || workspace_bytes < pl.ws_bytes) return RFSN_ERR_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return RFSN_ERR_ALIGNMENT;
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  pl.p.partial = reinterpret_cast<float*>(ws);
  pl.p.tickets = reinterpret_cast<unsigned*>(ws + pl.ctl_bytes);
  pl.p.dev_status = device_status;
  if ((st = encode_matrix(&pl.p.wmap, w, N, K, ldw, kLinTile)) != RFSN_OK) return st;
  if ((st = encode_matrix(&pl.p.xmap, x, M, K, ldx, kLinRows)) != RFSN_OK) return st;
  static bool smem_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !smem_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(rfsn_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLinSmem);
    if (e != cudaSuccess) return check_cuda(e);
    if (dev >= 0 && dev < 64) smem_set[dev] = true;
  }
  // programmatic dependent launch: the kernel may start while the previous kernel in the
  // stream finishes, and waits for it (griddepcontrol.wait) before reading its outputs
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.grid);
  cfg.blockDim = dim3(kLinThreads);
  cfg.dynamicSmemBytes = kLinSmem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, rfsn_linear_kernel, pl.p));
}
