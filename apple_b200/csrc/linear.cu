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
//   1  y = fp16(fp16(acc) + r)            the layer's residual add after o_proj / ffn_down
//   2  y = gelu_tanh(fp16(acc))           the layer's FFN activation, fp16 after every operation
//
// Work split.  W is cut into 64-row tiles and K into `splits` chunks; one work
// item is one (row tile, K chunk).  A persistent grid (one CTA per SM) deals the
// items round-robin.  In a CTA, a producer warp copies the item's W slab (64
// rows x kc) and x slab (M rows x kc) into a shared-memory ring with 1-D bulk
// copies (cp.async.bulk), one copy per row into a padded row (kc + 8 fp16), so
// that 8-row ldmatrix reads fall in distinct banks; the mbarriers that guard the
// stages are waited with bounds.  Eight consumer warps run mma.sync m16n8k16 on
// the slab: warp w owns output rows 16 (w / 4) .. + 16 and columns 16 (w % 4) ..
// + 16 of the tile.  Each item's fp32 partial tile goes to the workspace; the
// CTA that completes a row tile's last K chunk (a ticket per tile, tagged by a
// launch counter in the workspace as the decode-attention kernel does) sums the
// chunks in K order and applies the epilogue.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "rfsn_api_internal.h"
#include "rfsn_attn_util.cuh"
#include "rfsn_common.cuh"
#include "rfsn_elementwise.cuh"

namespace rfsn {

constexpr int kLinTile = 64;       // W rows per tile
constexpr int kLinRows = 32;       // activation rows (M <= 32)
constexpr int kLinConsumers = 8;   // consumer warps
constexpr int kLinMaxStages = 6;

struct LinParams {
  const uint16_t* x;   // [M][K] fp16, row stride ldx
  const uint16_t* w;   // [N][K] fp16, row stride ldw
  const uint16_t* r;   // epilogue 1: [M][N] fp16, row stride ldr
  uint16_t* y;         // [M][N] fp16, row stride ldy
  int64_t ldx, ldw, ldr, ldy;
  int M, N, K, kc, splits, epilogue;
  int items, stages, stage_bytes, x_off;  // x slab offset inside a stage
  int pitch;                              // padded slab row pitch in fp16 elements (kc + 8)
  float* partial;                         // [items][32][64] fp32
  unsigned long long* gen;                // [0] launch counter, [1] CTAs done
  unsigned long long* tickets;            // one per row tile
  int32_t* dev_status;
};

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

// Item i: row tile i / splits, K chunk i % splits (a tile's chunks are consecutive items).
__device__ __forceinline__ void item_coords(const LinParams& p, int i, int& tile, int& chunk) {
  tile = i / p.splits;
  chunk = i - tile * p.splits;
}

__global__ void __launch_bounds__((kLinConsumers + 1) * 32, 1) rfsn_linear_kernel(const __grid_constant__ LinParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kLinMaxStages;
  uint64_t* sync_bar = empty + kLinMaxStages;  // bounded barrier of the consumer warps
  volatile int* flags = reinterpret_cast<volatile int*>(sync_bar + 1);  // [0] abort, [1] tile done here
  unsigned char* ring = smem + 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row_bytes = (uint32_t)p.kc * 2;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLinConsumers);
    }
    mbar_init(sync_bar, kLinConsumers);
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  // activation rows past M are never copied: zero them once in every stage
  for (int s = 0; s < p.stages; ++s) {
    uint4* xr = reinterpret_cast<uint4*>(ring + (size_t)s * p.stage_bytes + p.x_off);
    const int per_row = p.pitch / 8;
    for (int i = p.M * per_row + threadIdx.x; i < kLinRows * per_row; i += blockDim.x) xr[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  unsigned long long tag = 0;
  if (threadIdx.x == 0) tag = *reinterpret_cast<volatile unsigned long long*>(p.gen) & kTagMask;

  if (warp == kLinConsumers) {  // ===== producer: one bulk copy per slab row =====
    int stage = 0;
    uint32_t phase = 0, inflight = 0, inflight_parity = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < p.items && ok; i += gridDim.x) {
      int tile, chunk;
      item_coords(p, i, tile, chunk);
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
      unsigned char* sb = ring + (size_t)stage * p.stage_bytes;
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)(kLinTile + p.M) * row_bytes);
      __syncwarp();  // the barrier is armed before any copy can complete
      const int64_t k0 = (int64_t)chunk * p.kc;
      for (int r = lane; r < kLinTile + p.M; r += 32) {
        if (r < kLinTile)
          bulk_g2s(sb + (size_t)r * p.pitch * 2, p.w + (int64_t)(tile * kLinTile + r) * p.ldw + k0, row_bytes,
                   &full[stage]);
        else
          bulk_g2s(sb + p.x_off + (size_t)(r - kLinTile) * p.pitch * 2, p.x + (int64_t)(r - kLinTile) * p.ldx + k0,
                   row_bytes, &full[stage]);
      }
      inflight |= 1u << stage;
      inflight_parity = (inflight_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (lane == 0 && !ok) {  // leave no copy writing into the CTA's shared memory
      for (int k = 0; k < p.stages; ++k) {
        if (!((inflight >> k) & 1u)) continue;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full[k], (inflight_parity >> k) & 1u))
          if (global_timer_ns() - t0 > kWaitLimitNs) break;
      }
    }
    return;
  }

  // ===== consumers: warp w computes rows 16 (w / 4) + [0, 16), columns 16 (w % 4) + [0, 16) of a tile =====
  const int mt = warp >> 2, nq = warp & 3;
  const int g = lane >> 2, t4 = lane & 3;
  const int a_row = 16 * mt + (lane & 15), a_col = (lane >> 4) * 8;
  const int b_row = 16 * nq + ((lane >> 4) << 3) + (lane & 7), b_col = ((lane >> 3) & 1) * 8;
  int stage = 0;
  uint32_t phase = 0, sync_phase = 0;
  for (int i = blockIdx.x; i < p.items; i += gridDim.x) {
    int tile, chunk;
    item_coords(p, i, tile, chunk);
    if (!mbar_wait_bounded(&full[stage], phase, flags)) {
      flags[0] = 1;
      if (p.dev_status) atomicExch(p.dev_status, kDevStatusTimeoutFull);
      break;
    }
    const uint16_t* sw = reinterpret_cast<const uint16_t*>(ring + (size_t)stage * p.stage_bytes);
    const uint16_t* sx = reinterpret_cast<const uint16_t*>(ring + (size_t)stage * p.stage_bytes + p.x_off);
    const uint16_t* ap = sx + (size_t)a_row * p.pitch + a_col;
    const uint16_t* bp = sw + (size_t)b_row * p.pitch + b_col;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
    for (int k = 0; k < p.kc; k += 16) {
      uint32_t a[4], b[4];
      ldsm_x4(a, ap + k);
      ldsm_x4(b, bp + k);
      mma16816(acc[0], a, b[0], b[1]);
      mma16816(acc[1], a, b[2], b[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);  // the slab is consumed
    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1u;
    }
    float* part = p.partial + (size_t)i * (kLinRows * kLinTile);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int col = 16 * nq + 8 * u + 2 * t4;
      *reinterpret_cast<float2*>(part + (16 * mt + g) * kLinTile + col) = make_float2(acc[u][0], acc[u][1]);
      *reinterpret_cast<float2*>(part + (16 * mt + g + 8) * kLinTile + col) = make_float2(acc[u][2], acc[u][3]);
    }
    __threadfence();  // the partial is visible device-wide before the tile's ticket is taken
    if (!lin_sync(sync_bar, sync_phase, flags)) break;
    if (threadIdx.x == 0) {
      const int tk = take_ticket(p.tickets + tile, tag, p.splits);
      if (tk < 0 && p.dev_status) atomicExch(p.dev_status, kDevStatusTicket);
      flags[1] = tk > 0;
    }
    if (!lin_sync(sync_bar, sync_phase, flags)) break;
    if (flags[1]) {  // this CTA completed the tile: sum its K chunks in order, then the epilogue
      __threadfence();
      const float* base = p.partial + (size_t)tile * p.splits * (kLinRows * kLinTile);
      for (int idx = threadIdx.x; idx < p.M * kLinTile; idx += kLinConsumers * 32) {
        const int m = idx / kLinTile, c = idx - m * kLinTile;
        float s = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) s = __fadd_rn(s, __ldcg(base + (size_t)sp * kLinRows * kLinTile + idx));
        const int64_t n = (int64_t)tile * kLinTile + c;
        uint16_t h = f2h(s);
        if (p.epilogue == 1) h = f2h(__fadd_rn(h2f(h), h2f(p.r[(int64_t)m * p.ldr + n])));
        else if (p.epilogue == 2) h = gelu_tanh_f16(h);
        p.y[(int64_t)m * p.ldy + n] = h;
      }
    }
  }
  // every CTA counts itself done; the last one resets that count and advances the launch counter
  if (threadIdx.x == 0) {
    if (atomicAdd(p.gen + 1, 1ull) == (unsigned long long)gridDim.x - 1ull) {
      atomicExch(p.gen + 1, 0ull);
      atomicAdd(p.gen, 1ull);
    }
  }
}

}  // namespace rfsn

namespace rfsn {

constexpr int kLinChunk = 256;  // K per work item

struct LinPlan {
  LinParams p;
  int grid;
  int64_t smem;
  size_t ws_bytes;
  int64_t ctl_bytes;
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
  p.x = x; p.w = w; p.r = r; p.y = y;
  p.ldx = ldx; p.ldw = ldw; p.ldr = ldr; p.ldy = ldy;
  p.M = M; p.N = N; p.K = K; p.kc = kLinChunk; p.splits = K / kLinChunk; p.epilogue = epilogue;
  const int64_t tiles = N / kLinTile;
  const int64_t items = tiles * p.splits;
  if (items >= (int64_t)1 << 30 || p.splits > 0xffff) return RFSN_ERR_UNSUPPORTED;
  p.items = (int)items;
  p.pitch = p.kc + 8;  // 16 bytes of padding: 8 consecutive rows of an ldmatrix read hit 8 bank groups
  p.x_off = kLinTile * p.pitch * 2;
  p.stage_bytes = (kLinTile + kLinRows) * p.pitch * 2;
  p.stages = 4;
  pl.smem = 256 + (int64_t)p.stages * p.stage_bytes;
  if (pl.smem > 227 * 1024) return RFSN_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  pl.grid = (int)(items < sms ? items : sms);
  pl.ctl_bytes = align_up(16 + tiles * 8, 256);
  pl.ws_bytes = (size_t)pl.ctl_bytes + (size_t)items * kLinRows * kLinTile * sizeof(float);
  return RFSN_OK;
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
  pl.p.gen = reinterpret_cast<unsigned long long*>(ws);
  pl.p.tickets = pl.p.gen + 2;
  pl.p.partial = reinterpret_cast<float*>(ws + pl.ctl_bytes);
  pl.p.dev_status = device_status;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaFuncSetAttribute(rfsn_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return check_cuda(e);
  rfsn_linear_kernel<<<pl.grid, (kLinConsumers + 1) * 32, pl.smem, s>>>(pl.p);
  return check_cuda(cudaGetLastError());
}
