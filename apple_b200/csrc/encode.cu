// encode.cu — spill encoder (hot -> warm/cold) and code -> fp16 decoder.
//
// rfsn_encode:  HybridQuantizerMLX.encode (quantization.py:305-308) per token:
//   PQ   (quantization.py:124-144): per subspace, fp32 d = |x|^2 - 2 x.c + |c|^2,
//        first arg-min, residual = fp16(x - c).
//   RVQ  (quantization.py:206-252): token active iff sqrt(sum r^2) > threshold;
//        for each layer, first arg-min over all Kr centroids (the reference's
//        512-wide chunks with a strict '<' merge select the same index),
//        running -= c in fp32.
//   sparse (extension): the S coordinates with the largest |x - decode(x)|
//        (ties to the lower index) keep fp16(x - decode(x)).
// One thread encodes one vector; codebooks are staged in shared memory and
// read as warp-wide broadcasts.  Distances use sequential fp32 sums; the
// reference's matmul summation order is unspecified, so codes can differ from
// it only where two candidates tie to fp32 rounding.
//
// rfsn_decode_codes: exact fp16 reconstruction (rfsn_decode.cuh) plus the
// sparse residual, one thread per (token, 8-dim group), 16-byte stores.
#include <cuda_runtime.h>

#include "rfsn_api_internal.h"
#include "rfsn_decode.cuh"
#include "rfsn_encode_tc.h"

namespace rfsn {

struct EncodeParams {
  const uint16_t* x;
  int64_t batch, tokens, heads, sb, st, sh;
  uint8_t* data;
  BlockLayout lay;
  int kv;
  int64_t cap, rows, slot, first;
  uint16_t* residual_out;
  const uint16_t* pq_cb;
  const uint16_t* rvq_cb;
  int M, K, ds, L, Kr, S, D, rvq_u16, rvq_smem;
  float thr;
};

constexpr int kEncThreads = 128;
constexpr int kMaxD = 128;

template <int D>
__global__ void __launch_bounds__(kEncThreads) encode_kernel(const __grid_constant__ EncodeParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint16_t* s_pq = reinterpret_cast<uint16_t*>(smem);                       // [M*K*ds]
  float* s_pqcc = reinterpret_cast<float*>(smem + align_up((int64_t)p.M * p.K * p.ds * 2, 16));  // [M*K]
  unsigned char* after_pq = reinterpret_cast<unsigned char*>(s_pqcc) + align_up((int64_t)p.M * p.K * 4, 16);
  float* s_rcc = reinterpret_cast<float*>(after_pq);                         // [L*Kr]
  uint16_t* s_rvq = reinterpret_cast<uint16_t*>(after_pq + align_up((int64_t)p.L * p.Kr * 4, 16));

  const int nthr = blockDim.x;
  // Stage codebooks and their squared norms (sequential fp32 sums; products of
  // fp16 values are exact in fp32, quantization.py:94).
  {
    const int n16 = p.M * p.K * p.ds / 8;
    for (int i = threadIdx.x; i < n16; i += nthr)
      reinterpret_cast<uint4*>(s_pq)[i] = reinterpret_cast<const uint4*>(p.pq_cb)[i];
    if (p.rvq_smem) {
      const int r16 = p.L * p.Kr * D / 8;
      for (int i = threadIdx.x; i < r16; i += nthr)
        reinterpret_cast<uint4*>(s_rvq)[i] = reinterpret_cast<const uint4*>(p.rvq_cb)[i];
    }
    for (int i = threadIdx.x; i < p.M * p.K; i += nthr) {
      const uint16_t* c = p.pq_cb + (size_t)i * p.ds;
      float s = 0.f;
      for (int k = 0; k < p.ds; ++k) {
        const float v = h2f(c[k]);
        s = __fmaf_rn(v, v, s);
      }
      s_pqcc[i] = s;
    }
    for (int i = threadIdx.x; i < p.L * p.Kr; i += nthr) {
      const uint16_t* c = p.rvq_cb + (size_t)i * D;
      float s = 0.f;
      for (int k = 0; k < D; ++k) {
        const float v = h2f(c[k]);
        s = __fmaf_rn(v, v, s);
      }
      s_rcc[i] = s;
    }
  }
  __syncthreads();

  const int64_t nvec = p.batch * p.tokens * p.heads;
  const int64_t v = (int64_t)blockIdx.x * nthr + threadIdx.x;
  if (v >= nvec) return;
  const int64_t h = v % p.heads;
  const int64_t t = (v / p.heads) % p.tokens;
  const int64_t b = v / (p.heads * p.tokens);
  const uint16_t* xs = p.x + b * p.sb + t * p.st + h * p.sh;

  uint16_t xh[D];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const uint4 w = reinterpret_cast<const uint4*>(xs)[i];
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xh[8 * i + 2 * k] = (uint16_t)(ww[k] & 0xffff);
      xh[8 * i + 2 * k + 1] = (uint16_t)(ww[k] >> 16);
    }
  }

  const int64_t row = b * p.heads + h;
  const int64_t tok = p.first + t;
  const int fk = p.kv * 5;
  uint8_t* f_pq = p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 0);
  uint8_t* f_rvq = p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 1);
  uint8_t* f_act = p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 2);
  uint8_t* f_spi = p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 3);
  uint16_t* f_spv = reinterpret_cast<uint16_t*>(p.data + field_byte(p.lay, p.rows, p.cap, p.slot, row, tok, fk + 4));

  // ---- PQ: per-subspace argmin, fp16 residual (quantization.py:133-142) ----
  uint8_t codes[kMaxD];
  float res[D];  // fp32 value of the fp16 residual
  for (int m = 0; m < p.M; ++m) {
    const int d0 = m * p.ds;
    float xx = 0.f;
    for (int k = 0; k < p.ds; ++k) {
      const float xv = h2f(xh[d0 + k]);
      xx = __fmaf_rn(xv, xv, xx);
    }
    float best = __int_as_float(0x7f800000);
    int bi = 0;
    const uint16_t* cb = s_pq + (size_t)m * p.K * p.ds;
    for (int c = 0; c < p.K; ++c) {
      float cross = 0.f;
      for (int k = 0; k < p.ds; ++k) cross = __fmaf_rn(h2f(xh[d0 + k]), h2f(cb[c * p.ds + k]), cross);
      const float d = __fadd_rn(__fsub_rn(xx, 2.0f * cross), s_pqcc[m * p.K + c]);
      if (d < best) {
        best = d;
        bi = c;
      }
    }
    codes[m] = (uint8_t)bi;
    for (int k = 0; k < p.ds; ++k) {
      const uint16_t r = f2h(__fsub_rn(h2f(xh[d0 + k]), h2f(cb[bi * p.ds + k])));
      res[d0 + k] = h2f(r);
      if (p.residual_out) p.residual_out[b * p.sb + t * p.st + h * p.sh + d0 + k] = r;
    }
  }
  // store PQ codes
  for (int m = 0; m < p.M; ++m) f_pq[m] = codes[m];

  // ---- RVQ (quantization.py:216-250) ----
  int rcodes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  bool active = false;
  if (p.L > 0) {
    float nn = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) nn = __fmaf_rn(res[i], res[i], nn);
    active = __fsqrt_rn(nn) > p.thr;
    if (active) {
      const uint16_t* rcb_all = p.rvq_smem ? s_rvq : p.rvq_cb;
      for (int l = 0; l < p.L; ++l) {
        float rr = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) rr = __fmaf_rn(res[i], res[i], rr);
        const uint16_t* rcb = rcb_all + (size_t)l * p.Kr * D;
        float best = __int_as_float(0x7f800000);
        int bi = 0;
        for (int c = 0; c < p.Kr; ++c) {
          const uint16_t* row_c = rcb + (size_t)c * D;
          float cross = 0.f;
#pragma unroll
          for (int i = 0; i < D; ++i) cross = __fmaf_rn(res[i], h2f(row_c[i]), cross);
          const float d = __fadd_rn(__fsub_rn(rr, 2.0f * cross), s_rcc[l * p.Kr + c]);
          if (d < best) {
            best = d;
            bi = c;
          }
        }
        if (l < 8) rcodes[l] = bi;
        const uint16_t* chosen = rcb + (size_t)bi * D;
#pragma unroll
        for (int i = 0; i < D; ++i) res[i] = __fsub_rn(res[i], h2f(chosen[i]));
        if (p.rvq_u16)
          reinterpret_cast<uint16_t*>(f_rvq)[l] = (uint16_t)bi;
        else
          f_rvq[l] = (uint8_t)bi;
      }
    } else {
      for (int l = 0; l < p.L; ++l) {
        if (p.rvq_u16)
          reinterpret_cast<uint16_t*>(f_rvq)[l] = 0;
        else
          f_rvq[l] = 0;
      }
    }
    f_act[0] = active ? 1 : 0;
  }

  // ---- sparse top-S residual (extension) ----
  if (p.S > 0) {
    QzView q;
    q.pq_cb = s_pq;
    q.rvq_cb = p.rvq_smem ? s_rvq : p.rvq_cb;
    q.M = p.M; q.K = p.K; q.ds = p.ds; q.L = p.L; q.Kr = p.Kr; q.D = D; q.S = p.S; q.rvq_u16 = p.rvq_u16;
    uint8_t rv8[8];
    uint16_t rv16[8];
    for (int l = 0; l < 8; ++l) {
      rv8[l] = (uint8_t)rcodes[l];
      rv16[l] = (uint16_t)rcodes[l];
    }
    const void* rvp = p.rvq_u16 ? (const void*)rv16 : (const void*)rv8;
    float err[D];
#pragma unroll
    for (int g = 0; g < D / 8; ++g) {
      uint32_t w[4];
      recon8(q, codes, rvp, active, 8 * g, w);
      float f[8];
      unpack8(w, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) err[8 * g + k] = __fsub_rn(h2f(xh[8 * g + k]), f[k]);
    }
    float mag[D];
#pragma unroll
    for (int i = 0; i < D; ++i) mag[i] = fabsf(err[i]);
    for (int s = 0; s < p.S; ++s) {
      float bm = -1.f;
      int bi = 0;
#pragma unroll
      for (int i = 0; i < D; ++i) {
        if (mag[i] > bm) {
          bm = mag[i];
          bi = i;
        }
      }
      float ev = 0.f;
#pragma unroll
      for (int i = 0; i < D; ++i) {
        if (i == bi) {
          ev = err[i];
          mag[i] = -2.f;
        }
      }
      f_spi[s] = (uint8_t)bi;
      f_spv[s] = f2h(ev);
    }
  }
}

struct DecodeCodesParams {
  QzView q;
  const uint8_t* data;
  BlockLayout lay;
  int kv;
  int64_t cap, store_rows, nrows, slot, first, count, heads;
  uint16_t* out;
  int64_t sb, st, sh;
};

__global__ void decode_codes_kernel(const __grid_constant__ DecodeCodesParams p) {
  const int G = p.q.D / 8;
  const int64_t total = p.nrows * p.count * G;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(i % G);
    const int64_t t = (i / G) % p.count;
    const int64_t row = i / ((int64_t)G * p.count);
    const int64_t tok = p.first + t;
    const int fk = p.kv * 5;
    const uint8_t* f_pq = p.data + field_byte(p.lay, p.store_rows, p.cap, p.slot, row, tok, fk + 0);
    const uint8_t* f_rvq = p.data + field_byte(p.lay, p.store_rows, p.cap, p.slot, row, tok, fk + 1);
    const uint8_t* f_act = p.data + field_byte(p.lay, p.store_rows, p.cap, p.slot, row, tok, fk + 2);
    const uint8_t* f_spi = p.data + field_byte(p.lay, p.store_rows, p.cap, p.slot, row, tok, fk + 3);
    const uint16_t* f_spv =
        reinterpret_cast<const uint16_t*>(p.data + field_byte(p.lay, p.store_rows, p.cap, p.slot, row, tok, fk + 4));
    const bool active = p.q.L > 0 && f_act[0] != 0;
    uint32_t w[4];
    recon8(p.q, f_pq, f_rvq, active, 8 * g, w);
    if (p.q.S > 0) {
      float f[8];
      unpack8(w, f);
      bool touched = false;
      for (int e = 0; e < p.q.S; ++e) {
        const int id = f_spi[e] - 8 * g;
        if (id >= 0 && id < 8) {
          touched = true;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (k == id) f[k] = __fadd_rn(f[k], h2f(f_spv[e]));
        }
      }
      if (touched) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const __half2 h2 = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
          w[k] = *reinterpret_cast<const uint32_t*>(&h2);
        }
      }
    }
    const int64_t b = row / p.heads, h = row % p.heads;
    uint4 o;
    o.x = w[0]; o.y = w[1]; o.z = w[2]; o.w = w[3];
    *reinterpret_cast<uint4*>(p.out + b * p.sb + t * p.st + h * p.sh + 8 * g) = o;
  }
}

}  // namespace rfsn

using namespace rfsn;

extern "C" int rfsn_encode(const rfsn_quantizer* qz, const uint16_t* x, int64_t batch, int64_t tokens, int64_t heads,
                           int64_t stride_b, int64_t stride_t, int64_t stride_h, const rfsn_code_store* dst,
                           int32_t kv, int64_t dst_slot, int64_t dst_first, uint16_t* residual_out, void* stream) {
  int st = validate_quantizer(qz);
  if (st != RFSN_OK) return st;
  if (!x || !dst || batch < 0 || tokens < 0 || heads <= 0) return RFSN_ERR_INVALID_ARGUMENT;
  if (qz->head_dim != 64 && qz->head_dim != 128) return RFSN_ERR_UNSUPPORTED;
  if (qz->rvq_layers > 8) return RFSN_ERR_UNSUPPORTED;
  st = validate_store(dst, qz);
  if (st != RFSN_OK) return st;
  if (batch * heads > dst->rows || dst_slot < 0 || dst_slot >= dst->slots || dst_first < 0 ||
      dst_first + tokens > dst->cap || (kv != 0 && kv != 1))
    return RFSN_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)x & 15) || (stride_b & 7) || (stride_t & 7) || (stride_h & 7)) return RFSN_ERR_ALIGNMENT;
  const int64_t nvec = batch * tokens * heads;
  if (nvec == 0) return RFSN_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // tensor-core encoder for the configurations it covers (bit-identical codes up to fp32 ties)
  if (encode_tc_supported(qz) && !((uintptr_t)residual_out & 15))
    return encode_tc_launch(qz, x, nullptr, batch, tokens, heads, stride_b, stride_t, stride_h, dst, kv, dst_slot,
                            dst_first, residual_out, s);

  EncodeParams p{};
  p.x = x; p.batch = batch; p.tokens = tokens; p.heads = heads;
  p.sb = stride_b; p.st = stride_t; p.sh = stride_h;
  p.data = dst->data; p.lay = layout_of(qz); p.kv = kv;
  p.cap = dst->cap; p.rows = dst->rows; p.slot = dst_slot; p.first = dst_first;
  p.residual_out = residual_out;
  p.pq_cb = qz->pq_codebooks; p.rvq_cb = qz->rvq_codebooks;
  p.M = qz->num_subspaces; p.K = qz->pq_codebook_size; p.ds = qz->subspace_dim; p.L = qz->rvq_layers;
  p.Kr = qz->rvq_codebook_size; p.S = qz->sparse_topk; p.D = qz->head_dim; p.rvq_u16 = qz->rvq_codebook_size > 256;
  p.thr = qz->rvq_threshold;
  const int64_t pq_bytes = align_up((int64_t)p.M * p.K * p.ds * 2, 16) + align_up((int64_t)p.M * p.K * 4, 16);
  const int64_t rcc_bytes = align_up((int64_t)p.L * p.Kr * 4, 16);
  const int64_t rvq_bytes = (int64_t)p.L * p.Kr * p.D * 2;
  int64_t smem = pq_bytes + rcc_bytes;
  p.rvq_smem = (smem + rvq_bytes) <= 160 * 1024;
  if (p.rvq_smem) smem += rvq_bytes;
  if (smem > 200 * 1024) return RFSN_ERR_UNSUPPORTED;
  const int blocks = (int)((nvec + kEncThreads - 1) / kEncThreads);
  cudaError_t e;
  if (p.D == 64) {
    e = cudaFuncSetAttribute(encode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) encode_kernel<64><<<blocks, kEncThreads, smem, s>>>(p);
  } else {
    e = cudaFuncSetAttribute(encode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) encode_kernel<128><<<blocks, kEncThreads, smem, s>>>(p);
  }
  return check_cuda(e == cudaSuccess ? cudaGetLastError() : e);
}

extern "C" int rfsn_encode_kv(const rfsn_quantizer* qz, const uint16_t* k, const uint16_t* v, int64_t batch,
                              int64_t tokens, int64_t heads, int64_t stride_b, int64_t stride_t, int64_t stride_h,
                              const rfsn_code_store* dst, int64_t dst_slot, int64_t dst_first, void* stream) {
  int st = validate_quantizer(qz);
  if (st != RFSN_OK) return st;
  if (!k || !v) return RFSN_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)v & 15)) return RFSN_ERR_ALIGNMENT;
  if (!encode_tc_supported(qz)) {  // two launches of the general encoder
    st = rfsn_encode(qz, k, batch, tokens, heads, stride_b, stride_t, stride_h, dst, 0, dst_slot, dst_first, nullptr,
                     stream);
    if (st != RFSN_OK) return st;
    return rfsn_encode(qz, v, batch, tokens, heads, stride_b, stride_t, stride_h, dst, 1, dst_slot, dst_first,
                       nullptr, stream);
  }
  // the K call's checks cover the shared shape, strides and destination
  if (!dst || batch < 0 || tokens < 0 || heads <= 0) return RFSN_ERR_INVALID_ARGUMENT;
  st = validate_store(dst, qz);
  if (st != RFSN_OK) return st;
  if (batch * heads > dst->rows || dst_slot < 0 || dst_slot >= dst->slots || dst_first < 0 ||
      dst_first + tokens > dst->cap)
    return RFSN_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)k & 15) || (stride_b & 7) || (stride_t & 7) || (stride_h & 7)) return RFSN_ERR_ALIGNMENT;
  if (batch * tokens * heads == 0) return RFSN_OK;
  return encode_tc_launch(qz, k, v, batch, tokens, heads, stride_b, stride_t, stride_h, dst, 0, dst_slot, dst_first,
                          nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int rfsn_decode_codes(const rfsn_quantizer* qz, const rfsn_code_store* src, int32_t kv, int64_t slot,
                                 int64_t first, int64_t count, int64_t batch, int64_t heads, uint16_t* out,
                                 int64_t stride_b, int64_t stride_t, int64_t stride_h, void* stream) {
  int st = validate_quantizer(qz);
  if (st != RFSN_OK) return st;
  if (!src || !out || count < 0 || batch < 0 || heads <= 0) return RFSN_ERR_INVALID_ARGUMENT;
  st = validate_store(src, qz);
  if (st != RFSN_OK) return st;
  if (batch * heads > src->rows || slot < 0 || slot >= src->slots || first < 0 || first + count > src->cap ||
      (kv != 0 && kv != 1))
    return RFSN_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)out & 15) || (stride_b & 7) || (stride_t & 7) || (stride_h & 7)) return RFSN_ERR_ALIGNMENT;
  if (count == 0 || batch == 0) return RFSN_OK;
  DecodeCodesParams p{};
  p.q.pq_cb = qz->pq_codebooks; p.q.rvq_cb = qz->rvq_codebooks;
  p.q.M = qz->num_subspaces; p.q.K = qz->pq_codebook_size; p.q.ds = qz->subspace_dim; p.q.L = qz->rvq_layers;
  p.q.Kr = qz->rvq_codebook_size; p.q.D = qz->head_dim; p.q.S = qz->sparse_topk;
  p.q.rvq_u16 = qz->rvq_codebook_size > 256;
  p.data = src->data; p.lay = layout_of(qz); p.kv = kv;
  p.cap = src->cap; p.store_rows = src->rows; p.nrows = batch * heads; p.slot = slot; p.first = first;
  p.count = count; p.heads = heads;
  p.out = out; p.sb = stride_b; p.st = stride_t; p.sh = stride_h;
  const int64_t total = batch * heads * count * (qz->head_dim / 8);
  const int threads = 256;
  const int64_t blocks64 = (total + threads - 1) / threads;
  const int blocks = (int)(blocks64 < 148 * 64 ? blocks64 : 148 * 64);
  decode_codes_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError());
}
