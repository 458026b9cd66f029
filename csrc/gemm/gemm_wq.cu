// Host launcher of the weight-only-quantised tcgen05 GEMM (Q4 block-32 / INT8 per row).
#include "../common/om_host.h"
#include "gemm_launch.h"
#include "gemm_wq.cuh"
#include "gemm_wq_dec.cuh"

namespace om {

template <int BX, int QT, bool SWAP>
static void launch_wq(const CUtensorMap& tx, const GemmArgs& g, int grid, cudaStream_t st) {
  using C = WqCfg<BX, QT, SWAP>;
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

template <int BX, int QT>
static void launch_dec(const CUtensorMap& tx, const GemmArgs& g, int grid, cudaStream_t st) {
  using C = WqDecCfg<BX, QT>;
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(gemm_wq_dec_kernel<BX, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES));
    attr_set[dev] = true;
  }
  gemm_wq_dec_kernel<BX, QT><<<grid, C::THREADS, C::SMEM_BYTES, st>>>(tx, g);
  OM_LAUNCH_CHECK();
}

template <int QT>
static void dispatch_dec(int bx, const CUtensorMap& tx, const GemmArgs& g, int grid, cudaStream_t st) {
  switch (bx) {
    case 32: return launch_dec<32, QT>(tx, g, grid, st);
    case 64: return launch_dec<64, QT>(tx, g, grid, st);
    default: return launch_dec<128, QT>(tx, g, grid, st);
  }
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
//    qtype 1, INT8: 8192-byte tiles = 128 rows x 64 offset-binary bytes);
// scales: INT8 only, fp32 [N] per-row scale (applied in the epilogue).
// Decode (M <= 256 tokens, with a workspace and the zeroed counters `sem`) runs the
// stream-K TMEM-operand kernel (gemm_wq_dec.cuh); larger M and prefill run the
// shared-memory-operand kernel (gemm_wq.cuh) with split-K planned by a byte model.
void om_gemm_wq(torch::Tensor x, torch::Tensor qtiles, c10::optional<torch::Tensor> scales, int64_t qtype,
                torch::Tensor out, c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> workspace,
                torch::Tensor status, int64_t force_swap, int64_t force_splits, std::vector<int64_t> peer,
                c10::optional<torch::Tensor> sem, std::vector<int64_t> agwait) {
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
  om::GemmArgs g{};
  om::PeerOut po;
  const bool has_peer = om::peer_from_list(peer, M, po);
  TORCH_CHECK(!has_peer || !resid.has_value(), "gemm_wq: peer output takes no residual");
  g.rows = rows;
  g.cols = cols;
  const int wt_tiles = (N + 127) / 128;  // 128-row weight tiles
  g.wt_tiles = wt_tiles;
  g.tiles_c = (cols + bn_mma - 1) / bn_mma;
  g.num_kb = K / 64;
  g.swap = swap ? 1 : 0;
  g.status = status.data_ptr<int>();
  g.ldo = out.stride(0);
  g.wscale = qtype == 1 ? scales->data_ptr<float>() : nullptr;
  g.wtiles = qtiles.data_ptr<uint8_t>();
  float* ws = nullptr;
  size_t ws_bytes = 0;
  if (workspace.has_value()) {
    TORCH_CHECK(workspace->is_cuda() && workspace->scalar_type() == at::kFloat && workspace->is_contiguous(),
                "gemm_wq: workspace must be contiguous fp32");
    ws = workspace->data_ptr<float>();
    ws_bytes = workspace->numel() * sizeof(float);
  }
  const __nv_bfloat16* rp = resid.has_value() ? reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr()) : nullptr;
  if (resid.has_value())
    TORCH_CHECK(resid->sizes() == out.sizes() && resid->stride(0) == out.stride(0), "gemm_wq: resid layout");
  TORCH_CHECK(x.stride(0) % 8 == 0, "gemm_wq: x row stride must be a multiple of 8 elements");
  auto st = at::cuda::getCurrentCUDAStream().stream();

  // ---------------------------------------------------------------- stream-K decode kernel
  const int dec_ch = qtype == 0 ? 4 : 2;
  const int dec_bx = std::min(bx, 128);
  const int dec_nh = (M + dec_bx - 1) / dec_bx;  // token halves (2 for 128 < M <= 256)
  const int dec_r = dec_bx == 32 ? 2 : 1;        // = WqDecCfg<dec_bx, *>::R
  if (swap && force_splits <= 0 && sem.has_value() && ws && g.num_kb % dec_ch == 0) {
    const int groups = (wt_tiles + dec_r - 1) / dec_r * dec_nh;
    const int nc = g.num_kb / dec_ch;
    const long long total = (long long)groups * nc;
    const int grid = (int)std::min<long long>(sms, total);
    const size_t part_bytes = (size_t)grid * 2 * dec_r * 128 * dec_bx * sizeof(float);
    TORCH_CHECK(part_bytes <= ws_bytes, "gemm_wq: workspace too small for the decode partials");
    TORCH_CHECK(sem->is_cuda() && sem->scalar_type() == at::kInt && sem->is_contiguous() && sem->numel() >= groups,
                "gemm_wq: sem must be zeroed int32 with one counter per row group");
    g.rgroup = dec_r;
    g.sk_total = total;
    g.sk_nc = nc;
    g.sk_nh = dec_nh;
    if (!agwait.empty()) {
      TORCH_CHECK(agwait.size() == 2 && agwait[0] != 0 && agwait[1] >= 1 && agwait[1] <= 8,
                  "gemm_wq: agwait = [own symmetric buffer, ranks]");
      g.agwait = reinterpret_cast<const int*>(agwait[0]);
      g.agwait_n = (int)agwait[1];
    }
    g.part = ws;
    g.sem = sem->data_ptr<int>();
    g.epi = rp ? om::EPI_RESID : om::EPI_STORE;
    g.out = out.data_ptr();
    g.resid = rp;
    if (has_peer) g.po = po;
    {
      bool v = (g.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0;
      if (rp) v = v && (reinterpret_cast<uintptr_t>(rp) & 15) == 0;
      if (has_peer) {
        v = v && (po.peer_off & 15) == 0;
        for (int i = 0; i < po.pworld; ++i) v = v && (reinterpret_cast<uintptr_t>(po.peer[i]) & 15) == 0;
      }
      g.vec_out = v ? 1 : 0;
    }
    // activations as [K/64][M][64]: a box {64, bx, ch} is `ch` swizzled [bx][64] tiles
    CUtensorMap tx = om::make_tmap_3d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, M, K / 64, x.stride(0),
                                      64, 64, dec_bx, dec_ch, CU_TENSOR_MAP_SWIZZLE_128B);
    if (qtype == 0)
      om::dispatch_dec<om::WQ_Q4>(dec_bx, tx, g, grid, st);
    else
      om::dispatch_dec<om::WQ_I8>(dec_bx, tx, g, grid, st);
    return;
  }

  TORCH_CHECK(agwait.empty(), "gemm_wq: agwait needs the decode kernel (M <= 256, workspace, sem)");
  // ---------------------------------------------------------------- shared-memory-operand kernel
  // Plan: choose the weight row-tiles per unit R (activation reuse, decode only) and
  // the split-K factor s by a byte-count model of the busiest SM: rounds of units x
  // bytes each unit streams (R packed weight tiles + one activation tile per kb), plus
  // the fp32 partials of split-K (written and re-read, spread over the SMs).
  int splits = 1, rgroup = 1;
  const int raw_bytes = tile_bytes;
  const int x_bytes = bx * 64 * 2;
  const int rmax = swap ? std::max(1, 256 / bn_mma) : 1;
  const bool can_split = ws && N % 4 == 0;
  const size_t max_split_ws = can_split ? std::max<size_t>(1, ws_bytes / ((size_t)M * N * sizeof(float))) : 1;
  if (force_splits > 0 && can_split) {
    splits = std::min<int>((int)force_splits, g.num_kb);
    rgroup = rmax;
    while (rgroup > 1 && (wt_tiles + rgroup - 1) / rgroup * g.tiles_c * splits < sms) rgroup >>= 1;
  } else {
    double best = 1e300;
    for (int R = 1; R <= rmax; R <<= 1) {
      const int groups = swap ? (wt_tiles + R - 1) / R : (rows + 127) / 128;
      for (int sc = 1; sc <= (can_split ? 16 : 1); ++sc) {
        if (sc > 1 && (g.num_kb / sc < 4 || (size_t)sc > max_split_ws)) break;
        const int kbps = (g.num_kb + sc - 1) / sc;
        const long long units = (long long)groups * g.tiles_c * sc;
        const long long rounds = (units + sms - 1) / sms;
        const double unit_bytes = (double)kbps * (std::min(R, wt_tiles) * raw_bytes + x_bytes);
        double cost = rounds * unit_bytes;
        if (sc > 1) cost += 2.0 * sc * (double)M * N * 4 / sms;
        if (cost < best * 0.98) {
          best = cost;
          splits = sc;
          rgroup = R;
        }
      }
    }
  }
  g.rgroup = swap ? rgroup : 1;
  g.tiles_r = swap ? (wt_tiles + g.rgroup - 1) / g.rgroup : (rows + 127) / 128;
  const int units = g.tiles_r * g.tiles_c;
  // copy chunk: the largest power of two <= the kernel's CHMAX dividing the K blocks
  int chunk = swap ? (bx <= 64 ? 4 : bx <= 128 ? 2 : 1) : 2;
  while (chunk > 1 && g.num_kb % chunk) chunk >>= 1;
  int kbps = (g.num_kb + splits - 1) / splits;
  kbps = (kbps + chunk - 1) / chunk * chunk;
  splits = (g.num_kb + kbps - 1) / kbps;
  g.chunk = chunk;
  g.splits = splits;
  g.kb_per_split = kbps;
  if (splits > 1) {
    g.epi = om::EPI_PARTIAL;
    g.out = ws;
    g.resid = nullptr;
  } else {
    g.epi = rp ? om::EPI_RESID : om::EPI_STORE;
    g.out = out.data_ptr();
    g.resid = rp;
    if (has_peer) g.po = po;
  }
  CUtensorMap tx = om::make_tmap_3d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, M, K / 64, x.stride(0), 64,
                                    64, bx, chunk, CU_TENSOR_MAP_SWIZZLE_128B);
  const int grid = std::min(units * splits, sms);
  if (qtype == 0)
    om::dispatch<om::WQ_Q4>(bx, swap, tx, g, grid, st);
  else
    om::dispatch<om::WQ_I8>(bx, swap, tx, g, grid, st);
  if (splits > 1)
    om::launch_splitk_reduce(ws, splits, M, N, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), rp,
                             qtype == 1 ? scales->data_ptr<float>() : nullptr, st, has_peer ? &po : nullptr);
}
