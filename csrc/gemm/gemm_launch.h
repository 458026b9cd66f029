// Launch-plan interface of the tcgen05 GEMM, shared by the dense and the
// weight-only-quantised launchers.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <vector>

namespace om {

struct PeerOut;

struct GemmPlan {
  int swap, bn, rows, cols, tiles_r, tiles_c, num_kb, splits, kb_per_split, grid;
};

GemmPlan plan_gemm(int M, int N, int K, int sms, bool allow_split, int force_swap);

void run_gemm(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int ldw, int M, int N, int K,
              __nv_bfloat16* out, int ldo, const __nv_bfloat16* resid, float* workspace, size_t ws_bytes,
              int* status, int force_swap, int force_splits, cudaStream_t st, const PeerOut* po = nullptr);

void launch_splitk_reduce(const float* ws, int splits, int M, int N, __nv_bfloat16* out, int ldo,
                          const __nv_bfloat16* resid, const float* col_scale, cudaStream_t st,
                          const PeerOut* po = nullptr);

// Peer-output descriptor from the Python-side list
// [partials byte offset, rows per rank, this rank, base pointer of rank 0, 1, ...];
// an empty list means local output. Returns false for the empty list.
bool peer_from_list(const std::vector<int64_t>& v, int M, PeerOut& po);

}  // namespace om
