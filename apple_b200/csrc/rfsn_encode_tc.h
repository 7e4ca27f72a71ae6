// rfsn_encode_tc.h — tensor-core spill encoder (encode_tc.cu), used by rfsn_encode
// for the configurations it covers; everything else runs encode.cu's kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rfsn_b200.h"

namespace rfsn {

// D = 64, 4- or 8-dim PQ subspaces, K <= 256 (multiple of 8), at most one RVQ
// layer with Kr <= 256 (multiple of 8).
bool encode_tc_supported(const rfsn_quantizer* qz);

// Same contract as rfsn_encode; x rows must be 16-byte aligned with strides in
// multiples of 8 elements.  With x_v non-null, one launch encodes x into the K
// fields (kv must be 0, no residual output) and x_v, laid out like x, into the V
// fields.
int encode_tc_launch(const rfsn_quantizer* qz, const uint16_t* x, const uint16_t* x_v, int64_t batch,
                     int64_t tokens, int64_t heads, int64_t sb, int64_t st, int64_t sh, const rfsn_code_store* dst,
                     int kv, int64_t slot, int64_t first, uint16_t* residual_out, cudaStream_t stream);

}  // namespace rfsn
