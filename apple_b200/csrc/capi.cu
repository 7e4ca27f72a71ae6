// capi.cu — version/status strings, validation helpers and cold-tier copies.
#include <cuda_runtime.h>
#include <string.h>

#include "rfsn_api_internal.h"
#include "rfsn_layout.h"

namespace {
thread_local char g_last_cuda_error[256] = "";
}

namespace rfsn {

int check_cuda(cudaError_t e) {
  if (e == cudaSuccess) return RFSN_OK;
  const char* s = cudaGetErrorString(e);
  strncpy(g_last_cuda_error, s ? s : "unknown CUDA error", sizeof(g_last_cuda_error) - 1);
  g_last_cuda_error[sizeof(g_last_cuda_error) - 1] = 0;
  return RFSN_ERR_CUDA;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate_quantizer(const rfsn_quantizer* qz) {
  if (!qz || !qz->pq_codebooks) return RFSN_ERR_INVALID_ARGUMENT;
  const int D = qz->head_dim, M = qz->num_subspaces, ds = qz->subspace_dim;
  if (D <= 0 || M <= 0 || ds <= 0 || M * ds != D || D % 8 != 0) return RFSN_ERR_INVALID_ARGUMENT;
  if (!(ds == 1 || ds == 2 || ds == 4 || ds % 8 == 0)) return RFSN_ERR_UNSUPPORTED;
  if (qz->pq_codebook_size <= 0 || qz->pq_codebook_size > 256) return RFSN_ERR_UNSUPPORTED;
  if (qz->rvq_layers < 0 || qz->sparse_topk < 0 || qz->sparse_topk > D) return RFSN_ERR_INVALID_ARGUMENT;
  if (qz->rvq_layers > 0) {
    if (!qz->rvq_codebooks || qz->rvq_codebook_size <= 0 || qz->rvq_codebook_size > 65536)
      return RFSN_ERR_INVALID_ARGUMENT;
    if (!aligned16(qz->rvq_codebooks)) return RFSN_ERR_ALIGNMENT;
  }
  if (!aligned16(qz->pq_codebooks)) return RFSN_ERR_ALIGNMENT;
  if (D > 255 && qz->sparse_topk > 0) return RFSN_ERR_UNSUPPORTED;  // uint8 sparse indices
  return RFSN_OK;
}

int validate_store(const rfsn_code_store* s, const rfsn_quantizer* qz) {
  (void)qz;
  if (!s || !s->data || s->cap <= 0 || s->rows <= 0 || s->slots <= 0) return RFSN_ERR_INVALID_ARGUMENT;
  if (s->cap % kBlockTokens != 0) return RFSN_ERR_ALIGNMENT;
  if (!aligned16(s->data)) return RFSN_ERR_ALIGNMENT;
  return RFSN_OK;
}

BlockLayout layout_of(const rfsn_quantizer* qz) {
  return make_block_layout(qz->num_subspaces, qz->rvq_layers, qz->rvq_codebook_size > 256, qz->sparse_topk);
}

}  // namespace rfsn

extern "C" int rfsn_version(void) { return RFSN_ABI_VERSION * 1000 + 1; }

extern "C" const char* rfsn_status_string(int status) {
  switch (status) {
    case RFSN_OK: return "ok";
    case RFSN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RFSN_ERR_UNSUPPORTED: return "unsupported configuration";
    case RFSN_ERR_CUDA: return "CUDA error";
    case RFSN_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case RFSN_ERR_DEVICE_TIMEOUT: return "device-side bounded wait timed out";
    case RFSN_ERR_ALIGNMENT: return "pointer, stride or capacity not 16-byte aligned";
    default: return "unknown status";
  }
}

extern "C" const char* rfsn_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" int64_t rfsn_code_block_bytes(const rfsn_quantizer* qz) {
  if (rfsn::validate_quantizer(qz) != RFSN_OK) return -1;
  return rfsn::layout_of(qz).block_bytes;
}

extern "C" int rfsn_cold_prefetch(void* dst_device, const void* src_pinned_host, size_t bytes, void* stream,
                                  void* event) {
  if ((!dst_device || !src_pinned_host) && bytes) return RFSN_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (bytes) {
    int st = rfsn::check_cuda(cudaMemcpyAsync(dst_device, src_pinned_host, bytes, cudaMemcpyHostToDevice, s));
    if (st != RFSN_OK) return st;
  }
  if (event) return rfsn::check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), s));
  return RFSN_OK;
}

extern "C" int rfsn_cold_evict(void* dst_pinned_host, const void* src_device, size_t bytes, void* stream) {
  if ((!dst_pinned_host || !src_device) && bytes) return RFSN_ERR_INVALID_ARGUMENT;
  if (!bytes) return RFSN_OK;
  return rfsn::check_cuda(cudaMemcpyAsync(dst_pinned_host, src_device, bytes, cudaMemcpyDeviceToHost,
                                          reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" int rfsn_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || !bytes) return RFSN_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  int st = rfsn::check_cuda(cudaMalloc(&p, bytes));
  if (st != RFSN_OK) return st;
  st = rfsn::check_cuda(cudaMemset(p, 0, bytes));
  if (st == RFSN_OK) {
    cudaIpcMemHandle_t h;
    st = rfsn::check_cuda(cudaIpcGetMemHandle(&h, p));
    if (st == RFSN_OK) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (st != RFSN_OK) {
    cudaFree(p);
    return st;
  }
  *ptr = p;
  return RFSN_OK;
}

extern "C" int rfsn_peer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return RFSN_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return rfsn::check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int rfsn_peer_close(void* ptr) {
  if (!ptr) return RFSN_ERR_INVALID_ARGUMENT;
  return rfsn::check_cuda(cudaIpcCloseMemHandle(ptr));
}

extern "C" int rfsn_peer_free(void* ptr) {
  if (!ptr) return RFSN_ERR_INVALID_ARGUMENT;
  return rfsn::check_cuda(cudaFree(ptr));
}
