// rfsn_api_internal.h — host-side validation and error plumbing shared by the C-ABI entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rfsn_b200.h"
#include "rfsn_layout.h"

namespace rfsn {

// Records the CUDA error text for rfsn_last_cuda_error() and maps it to a status.
int check_cuda(cudaError_t e);

// Checks the quantizer description: shapes, codebook pointers and alignment.
int validate_quantizer(const rfsn_quantizer* qz);

// Checks a code store: data present and 16-byte aligned, cap a multiple of 16.
int validate_store(const rfsn_code_store* s, const rfsn_quantizer* qz);

// Block layout of a code store for this quantizer.
BlockLayout layout_of(const rfsn_quantizer* qz);

}  // namespace rfsn
