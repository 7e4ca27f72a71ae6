// rfsn_layout.h — byte layout of one 16-token block of an rfsn_code_store.
//
// Field f = kv * 5 + k with k: 0 pq, 1 rvq, 2 active, 3 sp_idx, 4 sp_val.  Each
// field stores 16 tokens x bpt[k] bytes contiguously; absent fields take no
// space.  Host (planning, Python mirror in apple_b200/kernels.py) and device
// (encoder, decoder, fused attention) use this one definition.
#pragma once

#include <stdint.h>

namespace rfsn {

constexpr int kBlockTokens = 16;
constexpr int kNumFields = 10;  // K and V x {pq, rvq, active, sp_idx, sp_val}

struct BlockLayout {
  int off[kNumFields];  // byte offset of each field inside a block (0 when absent)
  int bpt[5];           // bytes per token of each field kind
  int block_bytes;
};

__host__ __device__ inline BlockLayout make_block_layout(int M, int L, int rvq_u16, int S) {
  BlockLayout b{};
  b.bpt[0] = M;
  b.bpt[1] = L * (rvq_u16 ? 2 : 1);
  b.bpt[2] = L > 0 ? 1 : 0;
  b.bpt[3] = S;
  b.bpt[4] = 2 * S;
  int off = 0;
  for (int f = 0; f < kNumFields; ++f) {
    b.off[f] = off;
    off += kBlockTokens * b.bpt[f % 5];
  }
  b.block_bytes = off;
  return b;
}

// Byte address of field f of token `tok` of row `row` in slot `slot`.
__host__ __device__ inline int64_t field_byte(const BlockLayout& b, int64_t rows, int64_t cap, int64_t slot,
                                              int64_t row, int64_t tok, int f) {
  const int64_t blk = ((slot * rows + row) * (cap / kBlockTokens)) + (tok / kBlockTokens);
  return blk * b.block_bytes + b.off[f] + (tok % kBlockTokens) * b.bpt[f % 5];
}

}  // namespace rfsn
