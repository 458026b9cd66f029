// Mixture-of-experts on the device, capturable in a CUDA graph (no host sync):
//
//   moe_route      router logits [T, E] -> top-k expert ids + softmax weights
//                  over the k selected logits (or weights for forced ids:
//                  Keep-Routing replay), per-expert counts
//   moe_permute    exclusive scan of the counts -> expert row offsets; every
//                  (token, slot) gets a row of the expert-sorted matrix and the
//                  token's activation row is copied there
//   grouped GEMM   Y_e = X_e @ W_e^T for all experts in one persistent tcgen05
//                  kernel (expert-sorted rows, stacked weights [E, N, K]); a work
//                  unit is (expert, 128-row tile, 128-col tile), found on the
//                  device from the offsets
//   moe_combine    out[t] (+)= sum_j w[t, j] * Y[row(t, j)]  (fp32 accumulate)
//
// Reference: MoE router top_k_selection + per-expert SwiGLU + weighted
// scatter-add (openmini-server/src/model/inference/model.rs:813-960, 1325;
// gguf.rs:1128-1336).
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"
#include "../gemm/gemm_tc.cuh"

namespace om {

constexpr int MOE_MAX_E = 256;
constexpr int MOE_MAX_K = 8;

// One warp per token: top-k by repeated warp argmax (ties -> lower expert id).
__global__ void moe_route_kernel(const __nv_bfloat16* __restrict__ logits, int T, int E, int k,
                                 const int* __restrict__ forced, int* __restrict__ ids, float* __restrict__ wts,
                                 int* __restrict__ counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const __nv_bfloat16* lg = logits + (size_t)warp * E;
  float sel[MOE_MAX_K];
  int sid[MOE_MAX_K];
  if (forced) {
    for (int j = 0; j < k; ++j) {
      sid[j] = min(max(forced[warp * k + j], 0), E - 1);
      sel[j] = __bfloat162float(lg[sid[j]]);
    }
  } else {
    constexpr int PER = MOE_MAX_E / 32;
    float v[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? __bfloat162float(lg[e]) : -INFINITY;
    }
    for (int j = 0; j < k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      sel[j] = bv;
      sid[j] = bi;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (lane + 32 * i == bi) v[i] = -INFINITY;
    }
  }
  if (lane == 0) {
    float mx = -INFINITY;
    for (int j = 0; j < k; ++j) mx = fmaxf(mx, sel[j]);
    float s = 0.f, p[MOE_MAX_K];
    for (int j = 0; j < k; ++j) {
      p[j] = __expf(sel[j] - mx);
      s += p[j];
    }
    for (int j = 0; j < k; ++j) {
      ids[warp * k + j] = sid[j];
      wts[warp * k + j] = p[j] / s;
      atomicAdd(&counts[sid[j]], 1);
    }
  }
}

// Single block: offsets = exclusive scan of counts (E <= 256); cursors reset.
__global__ void moe_scan_kernel(const int* __restrict__ counts, int E, int* __restrict__ offsets,
                                int* __restrict__ cursor) {
  __shared__ int s[MOE_MAX_E + 1];
  const int t = threadIdx.x;
  if (t < E) s[t] = counts[t];
  __syncthreads();
  if (t == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      const int c = s[e];
      s[e] = acc;
      acc += c;
    }
    s[E] = acc;
  }
  __syncthreads();
  if (t <= E) offsets[t] = s[t];
  if (t < E) cursor[t] = 0;
}

// One block per (token, slot): claim a row of its expert, copy the activation row there.
__global__ void moe_permute_kernel(const __nv_bfloat16* __restrict__ x, int D, const int* __restrict__ ids, int k,
                                   const int* __restrict__ offsets, int* __restrict__ cursor,
                                   int* __restrict__ row_of, __nv_bfloat16* __restrict__ xp) {
  const int tj = blockIdx.x;
  __shared__ int row;
  if (threadIdx.x == 0) {
    const int e = ids[tj];
    row = offsets[e] + atomicAdd(&cursor[e], 1);
    row_of[tj] = row;
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(tj / k) * D);
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)row * D);
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) dst[c] = src[c];
}

// out[t] = (resid[t] +) sum_j w[t, j] * yp[row_of[t, j]]
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ yp, int D, const int* __restrict__ row_of,
                                   const float* __restrict__ wts, int k, __nv_bfloat16* __restrict__ out,
                                   bool add_to_out) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
    float acc[8];
    if (add_to_out) {
      unpack8(reinterpret_cast<const uint4*>(out + (size_t)t * D)[c], acc);
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    }
    for (int j = 0; j < k; ++j) {
      const float w = wts[t * k + j];
      float y[8];
      unpack8(reinterpret_cast<const uint4*>(yp + (size_t)row_of[t * k + j] * D)[c], y);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += w * y[q];
    }
    reinterpret_cast<uint4*>(out + (size_t)t * D)[c] = pack8(acc);
  }
}

// ---------------------------------------------------------------- grouped GEMM
struct GroupedArgs {
  GemmArgs g;            // rows = total expert-sorted rows, cols = N, num_kb = K / 64
  const int* offsets;    // [E + 1] expert row offsets (device)
  int E;
  int N;                 // per-expert weight rows (weight tile y = e * N + n)
};

// unit -> (expert, 128-row tile, 128-col tile) using the per-expert tile prefix sums in smem
__device__ __forceinline__ bool grouped_unit(const int* cum, const int* offs, int E, int tiles_n, int u, int& e,
                                             int& mt, int& nt) {
  if (u >= cum[E]) return false;
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cum[mid] <= u) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int in = u - cum[e];
  mt = in / tiles_n;
  nt = in % tiles_n;
  return true;
}

__global__ void __launch_bounds__(256, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GroupedArgs ga) {
  constexpr int BN = 128;
  using C = GemmCfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  __shared__ int cum[MOE_MAX_E + 1];
  __shared__ int offs[MOE_MAX_E + 1];

  const GemmArgs& g = ga.g;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_n = (ga.N + BN - 1) / BN;
  for (int e = threadIdx.x; e <= ga.E; e += blockDim.x) offs[e] = ga.offsets[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < ga.E; ++e) {
      cum[e] = acc;
      acc += ((offs[e + 1] - offs[e] + 127) / 128) * tiles_n;
    }
    cum[ga.E] = acc;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, C::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      int e, mt, nt;
      for (int u = blockIdx.x; ok && grouped_unit(cum, offs, ga.E, tiles_n, u, e, mt, nt); u += gridDim.x) {
        const int row0 = offs[e] + mt * 128;
        for (int kb = 0; kb < g.num_kb; ++kb, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* a_dst = tiles + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(a_dst, &tmA, &full[s], kb * C::BK, row0);
          tma_load_2d(a_dst + C::A_BYTES, &tmB, &full[s], kb * C::BK, e * ga.N + nt * BN);
        }
      }
      if (!ok) {
        for (int j = max(0, it - C::STAGES); j < it; ++j)
          mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BN);
      int it = 0, local = 0;
      bool ok = true;
      int e, mt, nt;
      for (int u = blockIdx.x; ok && grouped_unit(cum, offs, ga.E, tiles_n, u, e, mt, nt);
           u += gridDim.x, ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&tempty[acc], ((local >> 1) & 1) ^ 1, g.status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < g.num_kb; ++kb, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(&full[s], (it / C::STAGES) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k)
            tc_mma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32, 1024), smem_desc_sw128(b_addr + k * 32, 1024), IDESC,
                       (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    int local = 0;
    int e, mt, nt;
    for (int u = blockIdx.x; grouped_unit(cum, offs, ga.E, tiles_n, u, e, mt, nt); u += gridDim.x, ++local) {
      const int acc = local & 1;
      if (!mbar_wait(&tfull[acc], (local >> 1) & 1, g.status, OM_ERR_WAIT_ACCUM)) break;
      tc_fence_after();
      GemmArgs gu = g;
      gu.rows = offs[e + 1];  // rows past this expert belong to the next one: not written
      const int r = offs[e] + mt * 128 + q * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + cc * 32, v);
        tc_wait_ld();
        epilogue_chunk(gu, v, r, nt * BN + cc * 32, 0);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace om

// ---------------------------------------------------------------- host entry points

// logits [T, E] bf16 -> ids [T, k] int32, weights [T, k] fp32, counts [E] int32 (zeroed here).
void om_moe_route(torch::Tensor logits, int64_t k, c10::optional<torch::Tensor> forced, torch::Tensor ids,
                  torch::Tensor wts, torch::Tensor counts) {
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.is_contiguous(), "moe_route: logits bf16");
  TORCH_CHECK(E <= om::MOE_MAX_E && k >= 1 && k <= om::MOE_MAX_K && k <= E, "moe_route: E <= 256, k <= 8");
  auto st = at::cuda::getCurrentCUDAStream().stream();
  OM_CUDA_CHECK(cudaMemsetAsync(counts.data_ptr(), 0, E * sizeof(int), st));
  if (T == 0) return;
  const int* fp = forced.has_value() ? forced->data_ptr<int>() : nullptr;
  om::moe_route_kernel<<<(T * 32 + 255) / 256, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), T, E, k, fp, ids.data_ptr<int>(),
      wts.data_ptr<float>(), counts.data_ptr<int>());
  OM_LAUNCH_CHECK();
}

// Expert-sorted copy of the activations: xp [T*k, D], row_of [T*k], offsets [E+1].
void om_moe_permute(torch::Tensor x, torch::Tensor ids, torch::Tensor counts, torch::Tensor offsets,
                    torch::Tensor cursor, torch::Tensor row_of, torch::Tensor xp) {
  const int T = x.size(0), D = x.size(1), k = ids.size(1), E = counts.numel();
  TORCH_CHECK(D % 8 == 0 && x.is_contiguous() && xp.is_contiguous(), "moe_permute: layouts");
  auto st = at::cuda::getCurrentCUDAStream().stream();
  om::moe_scan_kernel<<<1, 256 + 32, 0, st>>>(counts.data_ptr<int>(), E, offsets.data_ptr<int>(),
                                              cursor.data_ptr<int>());
  OM_LAUNCH_CHECK();
  if (T == 0) return;
  om::moe_permute_kernel<<<T * k, 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), D,
                                                ids.data_ptr<int>(), k, offsets.data_ptr<int>(),
                                                cursor.data_ptr<int>(), row_of.data_ptr<int>(),
                                                reinterpret_cast<__nv_bfloat16*>(xp.data_ptr()));
  OM_LAUNCH_CHECK();
}

// out [T, D] (+)= sum_j w[t, j] * yp[row_of[t, j]]
void om_moe_combine(torch::Tensor yp, torch::Tensor row_of, torch::Tensor wts, torch::Tensor out, bool add) {
  const int T = out.size(0), D = out.size(1), k = wts.size(1);
  TORCH_CHECK(D % 8 == 0 && yp.is_contiguous() && out.is_contiguous(), "moe_combine: layouts");
  if (T == 0) return;
  om::moe_combine_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(yp.data_ptr()), D, row_of.data_ptr<int>(), wts.data_ptr<float>(), k,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), add);
  OM_LAUNCH_CHECK();
}

// y [R, N] = x [R, K] (expert-sorted rows) @ w[e]^T, w: [E, N, K] bf16, offsets [E+1] on the device.
void om_grouped_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor offsets, torch::Tensor y, torch::Tensor status) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
              "grouped_gemm: bf16");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && y.is_contiguous() && w.dim() == 3, "grouped_gemm: layouts");
  const int R = x.size(0), K = x.size(1), E = w.size(0), N = w.size(1);
  TORCH_CHECK(w.size(2) == K && K % 64 == 0 && N % 8 == 0 && y.size(0) == R && y.size(1) == N,
              "grouped_gemm: shapes (K % 64, N % 8)");
  TORCH_CHECK(E <= om::MOE_MAX_E && offsets.numel() == E + 1, "grouped_gemm: offsets");
  if (R == 0) return;
  using C = om::GemmCfg<128>;
  om::GroupedArgs ga{};
  ga.g.rows = R;
  ga.g.cols = N;
  ga.g.num_kb = K / 64;
  ga.g.splits = 1;
  ga.g.kb_per_split = K / 64;
  ga.g.swap = 0;
  ga.g.epi = om::EPI_STORE;
  ga.g.out = y.data_ptr();
  ga.g.ldo = N;
  ga.g.status = status.data_ptr<int>();
  ga.offsets = offsets.data_ptr<int>();
  ga.E = E;
  ga.N = N;
  CUtensorMap ta = om::make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, R, K, 64, 128,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = om::make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, (uint64_t)E * N, K, 64, 128,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(om::grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES));
    attr_set[dev] = true;
  }
  om::grouped_gemm_kernel<<<om::num_sms(), 256, C::SMEM_BYTES, st>>>(ta, tb, ga);
  OM_LAUNCH_CHECK();
}
