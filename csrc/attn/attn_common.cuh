// Shared definitions of the paged attention kernels: partition size, launch
// arguments and the kernel that merges split-KV partial results.
#pragma once
#include "../common/om_ptx.cuh"

namespace om {

constexpr int ATT_PART = 512;  // keys per partition
constexpr int ATT_CHUNK = 128; // keys per inner iteration (one per thread)

struct AttnArgs {
  const __nv_bfloat16* q;  // [rows, ...] with per-row stride q_ld and head stride D
  int q_ld;
  const __nv_bfloat16* kc;  // [blocks, Hkv, 16, D]
  const __nv_bfloat16* vc;
  const int* block_tables;  // [S, max_blocks]
  int max_blocks;
  int num_seqs;             // S: rows of block_tables
  const int* row_seq;   // [rows] -> sequence index
  const int* row_ctx;   // [rows] -> number of visible keys
  __nv_bfloat16* out;   // [rows, Hq, D] with row stride out_ld
  int out_ld;
  float* part_o;        // [rows, Hq, NP, D]
  float* part_ml;       // [rows, Hq, NP, 2]
  int Hq, Hkv, NP;
  float scale_log2;     // softmax scale * log2(e)
  int num_blocks;
  int* status;
};

// Visible keys of `row`, checked against what the launch covers: a sequence index
// outside the block table, or a context longer than NP partitions or than the
// block-table row (max_blocks * 16 keys), records OM_ERR_BOUNDS and is clamped
// (context 0 for a bad sequence index, the covered maximum otherwise), so no
// kernel reads past the block table or silently drops keys.
__device__ __forceinline__ int checked_ctx(const AttnArgs& a, int row, int& seq) {
  int ctx = a.row_ctx[row];
  seq = a.row_seq[row];
  if (seq < 0 || seq >= a.num_seqs) {
    record_error(a.status, OM_ERR_BOUNDS);
    seq = 0;
    return 0;
  }
  const int cap = min(a.NP * ATT_PART, a.max_blocks * 16);
  if (ctx < 0 || ctx > cap) {
    record_error(a.status, OM_ERR_BOUNDS);
    ctx = ctx < 0 ? 0 : cap;
  }
  return ctx;
}

// Merge partitions: out = sum_p o_p 2^(m_p - M) / sum_p l_p 2^(m_p - M)
template <int D>
__global__ void attn_merge_kernel(const AttnArgs a) {
  const int row = blockIdx.x, h = blockIdx.y;
  int seq;
  const int ctx = checked_ctx(a, row, seq);
  const int np = min(a.NP, (ctx + ATT_PART - 1) / ATT_PART);
  const size_t base = ((size_t)row * a.Hq + h) * a.NP;
  float M = -INFINITY;
  for (int p = 0; p < np; ++p) M = fmaxf(M, a.part_ml[(base + p) * 2]);
  float L = 0.f;
  for (int p = 0; p < np; ++p) L += a.part_ml[(base + p) * 2 + 1] * exp2f(a.part_ml[(base + p) * 2] - M);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int p = 0; p < np; ++p) acc += a.part_o[(base + p) * D + d] * exp2f(a.part_ml[(base + p) * 2] - M);
    a.out[(size_t)row * a.out_ld + (size_t)h * D + d] = __float2bfloat16_rn(acc * inv);
  }
}

}  // namespace om
