// Host launchers for the tcgen05 GEMM: shape heuristics (swap-AB for decode,
// split-K when the tile count cannot fill 148 SMs), tensor-map encoding and
// the split-K reduction with its fused epilogue.
#include "../common/om_host.h"
#include "gemm_tc.cuh"
#include "gemm_launch.h"

namespace om {

// Sums the split-K partials, applies the optional per-column scale and
// residual, and stores bf16 rows locally or, with po.pworld > 0, into the
// owner rank's partials slot over NVLink followed by the epoch publication
// (the split-K form of the fused GEMM -> reduce-scatter).
__global__ void splitk_reduce_kernel(const float* __restrict__ P, int splits, int Ym, int Yn,
                                     __nv_bfloat16* __restrict__ Y, int ldo, const __nv_bfloat16* resid,
                                     const float* __restrict__ col_scale, const PeerOut po) {
  const size_t plane = (size_t)Ym * Yn;
  const int nv = Yn >> 2;  // float4 groups per row (Yn % 4 == 0 checked on host)
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)Ym * nv;
       i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / nv), n = (int)(i % nv) * 4;
    float4 acc = *reinterpret_cast<const float4*>(P + (size_t)m * Yn + n);
    for (int s = 1; s < splits; ++s) {
      float4 p = *reinterpret_cast<const float4*>(P + s * plane + (size_t)m * Yn + n);
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    __nv_bfloat16* y = (po.pworld > 0 ? peer_row(po, ldo, m) : Y + (size_t)m * ldo) + n;
    if (col_scale) {
      acc.x *= col_scale[n]; acc.y *= col_scale[n + 1]; acc.z *= col_scale[n + 2]; acc.w *= col_scale[n + 3];
    }
    if (resid) {
      const __nv_bfloat16* rr = resid + (size_t)m * ldo + n;
      uint2 rv = *reinterpret_cast<const uint2*>(rr);
      acc.x += bf16lo(rv.x); acc.y += bf16hi(rv.x); acc.z += bf16lo(rv.y); acc.w += bf16hi(rv.y);
    }
    uint2 o;
    o.x = pack_bf16x2(acc.x, acc.y);
    o.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(y) = o;
  }
  if (po.pworld > 0) {
    __threadfence_system();
    __syncthreads();
    peer_publish(po);
  }
}

template <int BN>
static void launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, int grid, cudaStream_t st) {
  using C = GemmCfg<BN>;
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES));
    attr_set[dev] = true;
  }
  gemm_bf16_tc_kernel<BN><<<grid, 256, C::SMEM_BYTES, st>>>(ta, tb, g);
  OM_LAUNCH_CHECK();
}

bool peer_from_list(const std::vector<int64_t>& v, int M, PeerOut& po) {
  po = PeerOut{};
  if (v.empty()) return false;
  const int world = (int)v.size() - 3;
  if (world < 1 || world > 8) throw std::runtime_error("peer output: 1..8 rank bases expected");
  po.peer_off = v[0];
  po.rows_own = (int)v[1];
  po.prank = (int)v[2];
  po.pworld = world;
  if (po.rows_own <= 0 || (long long)po.rows_own * world < M || po.prank < 0 || po.prank >= world ||
      po.peer_off % 16 != 0)
    throw std::runtime_error("peer output: bad rows_own / rank / offset");
  for (int i = 0; i < world; ++i) po.peer[i] = reinterpret_cast<uint8_t*>(v[3 + i]);
  return true;
}

GemmPlan plan_gemm(int M, int N, int K, int sms, bool allow_split, int force_swap) {
  GemmPlan p;
  p.swap = force_swap >= 0 ? force_swap : (M <= 128 ? 1 : 0);
  const int rows = p.swap ? N : M;
  const int cols = p.swap ? M : N;
  if (p.swap) {
    p.bn = cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : 256;
  } else {
    p.bn = cols <= 64 ? 64 : cols <= 128 ? 128 : 256;
  }
  p.rows = rows;
  p.cols = cols;
  p.tiles_r = (rows + 127) / 128;
  p.tiles_c = (cols + p.bn - 1) / p.bn;
  p.num_kb = (K + 63) / 64;
  const int units = p.tiles_r * p.tiles_c;
  p.splits = 1;
  if (allow_split && units < sms && (N % 4) == 0) {
    int s = std::max(1, std::min(p.num_kb, sms / units));
    if (s > 1) {
      int kbps = (p.num_kb + s - 1) / s;
      p.splits = (p.num_kb + kbps - 1) / kbps;
    }
  }
  p.kb_per_split = (p.num_kb + p.splits - 1) / p.splits;
  p.grid = std::min(units * p.splits, sms);
  return p;
}

static void set_splits(GemmPlan& p, int s, int sms) {
  s = std::max(1, std::min(s, p.num_kb));
  const int kbps = (p.num_kb + s - 1) / s;
  p.splits = (p.num_kb + kbps - 1) / kbps;
  p.kb_per_split = kbps;
  p.grid = std::min(p.tiles_r * p.tiles_c * p.splits, sms);
}

void run_gemm(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int ldw, int M, int N, int K,
              __nv_bfloat16* out, int ldo, const __nv_bfloat16* resid, float* workspace, size_t ws_bytes,
              int* status, int force_swap, int force_splits, cudaStream_t st, const PeerOut* po) {
  const int sms = num_sms();
  GemmPlan p = plan_gemm(M, N, K, sms, workspace != nullptr, force_swap);
  if (force_splits > 0 && workspace) set_splits(p, force_splits, sms);
  if (p.splits > 1 && (size_t)p.splits * M * N * sizeof(float) > ws_bytes)
    set_splits(p, (int)(ws_bytes / ((size_t)M * N * sizeof(float))), sms);  // as many splits as fit
  const __nv_bfloat16* a = p.swap ? w : x;
  const int lda = p.swap ? ldw : ldx;
  const __nv_bfloat16* b = p.swap ? x : w;
  const int ldb = p.swap ? ldx : ldw;
  CUtensorMap ta = make_tmap_2d(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, p.rows, lda, 64, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, p.cols, ldb, 64, p.bn,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  GemmArgs g{};
  g.rows = p.rows;
  g.cols = p.cols;
  g.num_kb = p.num_kb;
  g.splits = p.splits;
  g.kb_per_split = p.kb_per_split;
  g.tiles_r = p.tiles_r;
  g.tiles_c = p.tiles_c;
  g.swap = p.swap;
  g.status = status;
  g.ldo = ldo;
  g.wscale = nullptr;
  if (p.splits > 1) {
    g.epi = EPI_PARTIAL;
    g.out = workspace;
    g.resid = nullptr;
  } else {
    g.epi = resid ? EPI_RESID : EPI_STORE;
    g.out = out;
    g.resid = resid;
    if (po) g.po = *po;
  }
  switch (p.bn) {
    case 32: launch_bn<32>(ta, tb, g, p.grid, st); break;
    case 64: launch_bn<64>(ta, tb, g, p.grid, st); break;
    case 128: launch_bn<128>(ta, tb, g, p.grid, st); break;
    default: launch_bn<256>(ta, tb, g, p.grid, st); break;
  }
  if (p.splits > 1) launch_splitk_reduce(workspace, p.splits, M, N, out, ldo, resid, nullptr, st, po);
}

void launch_splitk_reduce(const float* ws, int splits, int M, int N, __nv_bfloat16* out, int ldo,
                          const __nv_bfloat16* resid, const float* col_scale, cudaStream_t st, const PeerOut* po) {
  const int nthreads = 256;
  const size_t work = (size_t)M * (N / 4);
  const int blocks = (int)std::min<size_t>((work + nthreads - 1) / nthreads, (size_t)num_sms() * 8);
  PeerOut pz{};
  splitk_reduce_kernel<<<blocks, nthreads, 0, st>>>(ws, splits, M, N, out, ldo, resid, col_scale, po ? *po : pz);
  OM_LAUNCH_CHECK();
}

}  // namespace om

// ------------------------------------------------------------------ torch op
void om_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> resid,
             c10::optional<torch::Tensor> workspace, torch::Tensor status, int64_t force_swap,
             int64_t force_splits, std::vector<int64_t> peer) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "om_gemm: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "om_gemm: bf16 tensors required");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "om_gemm: 2-D tensors");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "om_gemm: inner dim contiguous");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(0) == M && out.size(1) == N, "om_gemm: shape mismatch");
  TORCH_CHECK(K % 8 == 0, "om_gemm: K must be a multiple of 8");
  const __nv_bfloat16* rp = nullptr;
  if (resid.has_value()) {
    TORCH_CHECK(resid->sizes() == out.sizes() && resid->stride(0) == out.stride(0), "om_gemm: resid layout");
    rp = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
  }
  float* ws = nullptr;
  size_t ws_bytes = 0;
  if (workspace.has_value()) {
    ws = workspace->data_ptr<float>();
    ws_bytes = workspace->numel() * sizeof(float);
  }
  om::PeerOut po;
  const bool has_peer = om::peer_from_list(peer, M, po);
  TORCH_CHECK(!has_peer || !resid.has_value(), "om_gemm: peer output takes no residual");
  if (M == 0) return;
  om::run_gemm(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
               reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), w.stride(0), M, N, K,
               reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), rp, ws, ws_bytes,
               status.data_ptr<int>(), (int)force_swap, (int)force_splits,
               at::cuda::getCurrentCUDAStream().stream(), has_peer ? &po : nullptr);
}

std::vector<int64_t> om_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t sms, bool allow_split) {
  om::GemmPlan p = om::plan_gemm(M, N, K, sms, allow_split, -1);
  return {p.swap, p.bn, p.tiles_r, p.tiles_c, p.splits, p.kb_per_split, p.grid};
}
