// route.cu — centroid routing of the cold tier: chunk scores and their top-k.
//
// The reference's router picks cold chunks by distance from the current
// position (storage.py:166-182) and the cache then decodes every cold chunk the
// window overlaps (cache.py:293-342).  The routed mode of the B200 build
// instead attends only the k cold chunks whose key centroid (the mean of the
// chunk's decoded keys, per row) scores highest against the step's queries:
//
//   score[c] = max over sequences b, queries i and query heads h of
//              q[b, i, h] . centroid[c][b * kv_heads + h / group]
//
// one score per chunk for the whole batch (every row shares the chunk ids).
// A dot product is 32 lane-strided fp32 FMA chains combined by a fixed
// butterfly of fp32 adds.  The top k are ordered by descending score, ties to
// the lower chunk index.
#include <cuda_runtime.h>
#include <float.h>

#include "rfsn_api_internal.h"
#include "rfsn_common.cuh"

namespace rfsn {

constexpr int kRouteThreads = 256;
constexpr int kRouteMaxK = 64;

// One CTA per chunk: each warp takes (b, i, h) triples, the CTA keeps the max.
__global__ void __launch_bounds__(kRouteThreads) route_score_kernel(const uint16_t* q, int64_t q_bstride,
                                                                    const float* cent, int B, int Q, int Hq, int Hkv,
                                                                    int D, float* scores) {
  __shared__ float s_max[kRouteThreads / 32];
  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = Hq / Hkv;
  const int rows = B * Hkv;
  float best = -FLT_MAX;
  for (int t = warp; t < B * Q * Hq; t += kRouteThreads / 32) {
    const int b = t / (Q * Hq), r = t - b * Q * Hq, i = r / Hq, h = r - i * Hq;
    const uint16_t* qv = q + (size_t)b * q_bstride + ((size_t)i * Hq + h) * D;
    const float* cv = cent + ((size_t)c * rows + (size_t)b * Hkv + h / G) * D;
    // lane-strided partial dots, then a fixed-order tree: the same order for every triple
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s = __fmaf_rn(h2f(qv[d]), cv[d], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    best = fmaxf(best, s);
  }
  if (lane == 0) s_max[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = s_max[0];
    for (int w = 1; w < kRouteThreads / 32; ++w) m = fmaxf(m, s_max[w]);
    scores[c] = m;
  }
}

// One CTA: k rounds of a block-wide (max score, min index) over the untaken chunks.
__global__ void __launch_bounds__(kRouteThreads) route_topk_kernel(const float* scores, int C, int k, int32_t* ids,
                                                                   unsigned char* taken) {
  __shared__ float s_v[kRouteThreads / 32];
  __shared__ int s_i[kRouteThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < C; c += kRouteThreads) taken[c] = 0;
  __syncthreads();
  for (int round = 0; round < k; ++round) {
    float v = -FLT_MAX;
    int idx = 0x7fffffff;
    for (int c = threadIdx.x; c < C; c += kRouteThreads) {
      const float s = fmaxf(scores[c], -FLT_MAX);  // NaN and -inf rank with the lowest finite score
      if (!taken[c] && (s > v || (s == v && c < idx))) {
        v = s;
        idx = c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      if (v2 > v || (v2 == v && i2 < idx)) {
        v = v2;
        idx = i2;
      }
    }
    if (lane == 0) {
      s_v[warp] = v;
      s_i[warp] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bv = s_v[0];
      int bi = s_i[0];
      for (int w = 1; w < kRouteThreads / 32; ++w)
        if (s_v[w] > bv || (s_v[w] == bv && s_i[w] < bi)) {
          bv = s_v[w];
          bi = s_i[w];
        }
      ids[round] = bi;
      taken[bi] = 1;
    }
    __syncthreads();
  }
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_route_topk(const uint16_t* q, int64_t q_batch_stride, int32_t batch, int32_t queries,
                               int32_t q_heads, int32_t kv_heads, int32_t head_dim, const float* centroids,
                               int32_t num_chunks, int32_t k, float* scores, int32_t* ids, uint8_t* scratch,
                               void* stream) {
  if (!q || !centroids || !scores || !ids || !scratch) return RFSN_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || queries <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || q_heads % kv_heads)
    return RFSN_ERR_INVALID_ARGUMENT;
  if (num_chunks < 0 || k < 0 || k > num_chunks || k > kRouteMaxK) return RFSN_ERR_INVALID_ARGUMENT;
  const int64_t packed = (int64_t)queries * q_heads * head_dim;
  if (q_batch_stride != 0 && q_batch_stride < packed) return RFSN_ERR_INVALID_ARGUMENT;
  if (num_chunks == 0 || k == 0) return RFSN_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  route_score_kernel<<<num_chunks, kRouteThreads, 0, s>>>(q, q_batch_stride ? q_batch_stride : packed, centroids,
                                                         batch, queries, q_heads, kv_heads, head_dim, scores);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e);
  route_topk_kernel<<<1, kRouteThreads, 0, s>>>(scores, num_chunks, k, ids, scratch);
  return check_cuda(cudaGetLastError());
}
