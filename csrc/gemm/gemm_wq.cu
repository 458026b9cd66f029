// Host launcher of the weight-only-quantised tcgen05 GEMM (Q4 block-32 / INT8 per row).
#include "../common/om_host.h"
#include "gemm_launch.h"
#include "gemm_wq.cuh"

namespace om {

template <int BX, int QT, bool SWAP>
static void launch_wq(const CUtensorMap& tx, const GemmArgs& g, int grid, cudaStream_t st) {
  using C = WqCfg<BX, QT>;
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(gemm_wq_tc_kernel<BX, QT, SWAP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES));
    attr_set[dev] = true;
  }
  gemm_wq_tc_kernel<BX, QT, SWAP><<<grid, 512, C::SMEM_BYTES, st>>>(tx, g);
  OM_LAUNCH_CHECK();
}

template <int QT>
static void dispatch(int bx, bool swap, const CUtensorMap& tx, const GemmArgs& g, int grid, cudaStream_t st) {
  if (!swap) return launch_wq<128, QT, false>(tx, g, grid, st);
  switch (bx) {
    case 32: return launch_wq<32, QT, true>(tx, g, grid, st);
    case 64: return launch_wq<64, QT, true>(tx, g, grid, st);
    case 128: return launch_wq<128, QT, true>(tx, g, grid, st);
    default: return launch_wq<256, QT, true>(tx, g, grid, st);
  }
}

}  // namespace om

// Weight-only quantised GEMM: out[M, N] = x[M, K] @ dequant(W)^T (+ resid).
// qtiles: uint8 [ceil(N/128), K/64, tile bytes] in the tiled device format
//   (qtype 0, Q4: 4608-byte tiles = 128 rows x 32 B nibbles + [2][128] bf16 scales;
//    qtype 1, INT8: 8192-byte tiles = 128 rows x 64 B);
// scales: INT8 only, fp32 [N] per-row scale (applied in the epilogue).
void om_gemm_wq(torch::Tensor x, torch::Tensor qtiles, c10::optional<torch::Tensor> scales, int64_t qtype,
                torch::Tensor out, c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> workspace,
                torch::Tensor status, int64_t force_swap, int64_t force_splits) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "gemm_wq: x");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.dim() == 2, "gemm_wq: out");
  const int M = x.size(0), K = x.size(1), N = out.size(1);
  TORCH_CHECK(out.size(0) == M, "gemm_wq: out shape");
  TORCH_CHECK(K % 64 == 0, "gemm_wq: K must be a multiple of 64");
  const int tile_bytes = qtype == 0 ? 4608 : 8192;
  TORCH_CHECK(qtiles.is_contiguous() && qtiles.scalar_type() == at::kByte && qtiles.dim() == 3 &&
                  qtiles.size(0) == (N + 127) / 128 && qtiles.size(1) == K / 64 && qtiles.size(2) == tile_bytes,
              "gemm_wq: qtiles must be uint8 [ceil(N/128), K/64, ", tile_bytes, "]");
  if (qtype == 1)
    TORCH_CHECK(scales.has_value() && scales->scalar_type() == at::kFloat && scales->numel() == N,
                "gemm_wq: INT8 needs fp32 per-row scales");
  if (M == 0) return;
  const int sms = om::num_sms();
  const bool swap = force_swap >= 0 ? force_swap != 0 : M <= 256;
  TORCH_CHECK(!swap || M <= 256, "gemm_wq: swap mode needs M <= 256");
  const int rows = swap ? N : M, cols = swap ? M : N;
  const int bx = swap ? (M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256) : 128;
  const int bn_mma = swap ? bx : 128;
  om::GemmArgs g;
  g.rows = rows;
  g.cols = cols;
  g.tiles_r = (rows + 127) / 128;
  g.tiles_c = (cols + bn_mma - 1) / bn_mma;
  g.num_kb = K / 64;
  const int units = g.tiles_r * g.tiles_c;
  int splits = 1;
  float* ws = nullptr;
  size_t ws_bytes = 0;
  if (workspace.has_value()) {
    ws = workspace->data_ptr<float>();
    ws_bytes = workspace->numel() * sizeof(float);
  }
  if (ws && N % 4 == 0) {
    if (force_splits > 0) {
      splits = (int)force_splits;
    } else {
      // smallest split count whose work units fill the persistent grid's rounds
      // to within 6% (each split keeps >= 8 K blocks)
      double best = 1e30;
      for (int s = 1; s <= 16 && g.num_kb / s >= 8; ++s) {
        const int u = units * s;
        const double rounds = (double)((u + sms - 1) / sms);
        const double waste = rounds * sms / u;
        if (waste < best * 0.94) {
          best = waste;
          splits = s;
        }
      }
    }
    splits = std::min<int>(splits, g.num_kb);
    splits = std::min<int>(splits, (int)std::max<size_t>(1, ws_bytes / ((size_t)M * N * sizeof(float))));
  }
  const int kbps = (g.num_kb + splits - 1) / splits;
  splits = (g.num_kb + kbps - 1) / kbps;
  g.splits = splits;
  g.kb_per_split = kbps;
  g.swap = swap ? 1 : 0;
  g.status = status.data_ptr<int>();
  g.ldo = out.stride(0);
  g.wscale = qtype == 1 ? scales->data_ptr<float>() : nullptr;
  g.wtiles = qtiles.data_ptr<uint8_t>();
  const __nv_bfloat16* rp = resid.has_value() ? reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr()) : nullptr;
  if (resid.has_value())
    TORCH_CHECK(resid->sizes() == out.sizes() && resid->stride(0) == out.stride(0), "gemm_wq: resid layout");
  if (splits > 1) {
    g.epi = om::EPI_PARTIAL;
    g.out = ws;
    g.resid = nullptr;
  } else {
    g.epi = rp ? om::EPI_RESID : om::EPI_STORE;
    g.out = out.data_ptr();
    g.resid = rp;
  }
  CUtensorMap tx = om::make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, x.stride(0), 64, bx,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  const int grid = std::min(units * splits, sms);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (qtype == 0)
    om::dispatch<om::WQ_Q4>(bx, swap, tx, g, grid, st);
  else
    om::dispatch<om::WQ_I8>(bx, swap, tx, g, grid, st);
  if (splits > 1)
    om::launch_splitk_reduce(ws, splits, M, N, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), rp,
                             qtype == 1 ? scales->data_ptr<float>() : nullptr, st);
}
