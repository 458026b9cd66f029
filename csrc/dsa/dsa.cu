// Dynamic Sparse Attention (DSA) kernels.
//
//   1. indexer scores   I(t, s) = sum_h w_h(t) * relu(q_h(t) . k(s))   over the
//                       paged indexer-key cache (H_I heads x 64 dims per query,
//                       one 64-dim key per token), causal (s < ctx(t))
//   2. top-k            per query row, the k highest-scoring key positions
//                       (threshold by bitwise binary search over order-preserving
//                       keys held in shared memory, then an ordered compaction)
//   3. sparse attention softmax attention of each query row over its selected
//                       keys only, gathered from the paged K/V cache, GQA
//
// The reference's DSA (openmini-server/src/model/inference/dsa.rs:315-345,
// 761-824, 1321-1488) uses the full Q.K^T of all heads as its "indexer" and
// sorts; here the indexer is the lightweight multi-head ReLU scorer of the
// benchmark configuration and selection is sort-free.
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

constexpr int DSA_DIM = 64;
constexpr int DSA_MAX_HEADS = 8;

// grid (rows, ceil(max_ctx / 256)), 256 threads: thread = key
__global__ void dsa_scores_kernel(const __nv_bfloat16* __restrict__ qi, int q_ld, const float* __restrict__ wi,
                                  int w_ld, int H, const __nv_bfloat16* __restrict__ icache,
                                  const int* __restrict__ bt, int max_blocks, const int* __restrict__ row_seq,
                                  const int* __restrict__ row_ctx, float* __restrict__ scores, int s_ld,
                                  int num_blocks, int* status) {
  __shared__ float qs[DSA_MAX_HEADS][DSA_DIM];
  __shared__ float ws[DSA_MAX_HEADS];
  const int row = blockIdx.x;
  const int ctx = row_ctx[row];
  const int key = blockIdx.y * blockDim.x + threadIdx.x;
  for (int i = threadIdx.x; i < H * DSA_DIM; i += blockDim.x)
    qs[i / DSA_DIM][i % DSA_DIM] = __bfloat162float(qi[(size_t)row * q_ld + i]);
  if (threadIdx.x < H) ws[threadIdx.x] = wi[(size_t)row * w_ld + threadIdx.x];
  __syncthreads();
  if (key >= s_ld) return;
  if (key >= ctx) {
    scores[(size_t)row * s_ld + key] = -INFINITY;
    return;
  }
  int blk = bt[(size_t)row_seq[row] * max_blocks + (key >> 4)];
  if (blk < 0 || blk >= num_blocks) {
    record_error(status, OM_ERR_BOUNDS);
    blk = 0;
  }
  const uint4* kr = reinterpret_cast<const uint4*>(icache + ((size_t)blk * 16 + (key & 15)) * DSA_DIM);
  float acc[DSA_MAX_HEADS];
#pragma unroll
  for (int h = 0; h < DSA_MAX_HEADS; ++h) acc[h] = 0.f;
#pragma unroll
  for (int v = 0; v < DSA_DIM / 8; ++v) {
    const uint4 u = kr[v];
    const float k8[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                         bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
    for (int h = 0; h < DSA_MAX_HEADS; ++h) {
      if (h < H) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[h] += qs[h][v * 8 + j] * k8[j];
      }
    }
  }
  float s = 0.f;
#pragma unroll
  for (int h = 0; h < DSA_MAX_HEADS; ++h)
    if (h < H) s += ws[h] * fmaxf(acc[h], 0.f);
  scores[(size_t)row * s_ld + key] = s;
}

// Head reduction after the tensor-core indexer GEMM. g [rows * H, g_ld] bf16 holds
// q_h(t) . k(s) for the rows of one sequence segment (head-minor) over its first S
// keys; scores[r][s] = sum_h w[r][h] relu(g[r H + h][s]) for s < ctx_r, -inf for
// ctx_r <= s < s_ld. grid (ceil(s_ld / 1024), rows), 128 threads x 8 keys.
__global__ void __launch_bounds__(128) dsa_head_reduce_kernel(const __nv_bfloat16* __restrict__ g, int g_ld, int S,
                                                               const float* __restrict__ w, int w_ld, int H,
                                                               const int* __restrict__ row_ctx,
                                                               float* __restrict__ scores, int s_ld) {
  const int r = blockIdx.y;
  const int s0 = (blockIdx.x * 128 + threadIdx.x) * 8;
  if (s0 >= s_ld) return;
  const int ctx = min(row_ctx[r], S);
  float wr[DSA_MAX_HEADS];
#pragma unroll
  for (int h = 0; h < DSA_MAX_HEADS; ++h) wr[h] = h < H ? w[(size_t)r * w_ld + h] : 0.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (s0 + 8 <= S) {
#pragma unroll
    for (int h = 0; h < DSA_MAX_HEADS; ++h) {
      if (h >= H) break;
      const uint4 u = *reinterpret_cast<const uint4*>(g + ((size_t)r * H + h) * g_ld + s0);
      const float v[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                          bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += wr[h] * fmaxf(v[j], 0.f);
    }
  } else {
    for (int h = 0; h < H; ++h)
      for (int j = 0; j < 8 && s0 + j < S; ++j)
        acc[j] += wr[h] * fmaxf(__bfloat162float(g[((size_t)r * H + h) * g_ld + s0 + j]), 0.f);
  }
  float* out = scores + (size_t)r * s_ld + s0;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (s0 + j < s_ld) out[j] = s0 + j < ctx ? acc[j] : -INFINITY;
}

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// One CTA (1024 threads) per row. Selects min(k, ctx) positions with the
// highest scores; ties at the threshold are taken in increasing position
// order. out_idx [rows, k] (unused tail = -1), out_n [rows].
__global__ void __launch_bounds__(1024) dsa_topk_kernel(const float* __restrict__ scores, int s_ld,
                                                        const int* __restrict__ row_ctx, int k,
                                                        int* __restrict__ out_idx, int* __restrict__ out_n) {
  extern __shared__ uint32_t keys[];  // [s_ld]
  __shared__ int red[33];
  __shared__ int base_gt, base_eq;
  const int row = blockIdx.x;
  const int ctx = min(row_ctx[row], s_ld);
  const int kk = min(k, ctx);
  for (int i = threadIdx.x; i < ctx; i += blockDim.x) keys[i] = fkey(scores[(size_t)row * s_ld + i]);
  __syncthreads();
  auto count_ge = [&](uint32_t t) {
    int c = 0;
    for (int i = threadIdx.x; i < ctx; i += blockDim.x) c += keys[i] >= t;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
      int s = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
      red[32] = s;
    }
    __syncthreads();
    return red[32];
  };
  uint32_t thr = 0;
  if (kk < ctx) {
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = thr | (1u << bit);
      if (count_ge(cand) >= kk) thr = cand;
    }
  }
  // ordered compaction: all keys > thr first (they fit), then keys == thr until k
  if (threadIdx.x == 0) {
    base_gt = 0;
    base_eq = 0;
  }
  __syncthreads();
  const int n_gt = kk < ctx ? count_ge(thr + 1u) : 0;
  int* dst = out_idx + (size_t)row * k;
  // block-wide ordered scan over chunks of blockDim keys
  for (int c0 = 0; c0 < ctx; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    const uint32_t key = i < ctx ? keys[i] : 0u;
    const bool gt = i < ctx && (kk == ctx || key > thr);
    const bool eq = i < ctx && kk < ctx && key == thr;
    // warp ballots -> per-warp prefix
    const uint32_t bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __shared__ int wg[32], we[32];
    if (lane == 0) {
      wg[w] = __popc(bg);
      we[w] = __popc(be);
    }
    __syncthreads();
    int pg = 0, pe = 0;
    for (int j = 0; j < w; ++j) {
      pg += wg[j];
      pe += we[j];
    }
    const uint32_t lm = (1u << lane) - 1u;
    if (gt) dst[base_gt + pg + __popc(bg & lm)] = i;
    if (eq) {
      const int slot = base_eq + pe + __popc(be & lm);
      if (n_gt + slot < kk) dst[n_gt + slot] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int tg = 0, te = 0;
      for (int j = 0; j < (int)(blockDim.x >> 5); ++j) {
        tg += wg[j];
        te += we[j];
      }
      base_gt += tg;
      base_eq += te;
    }
    __syncthreads();
  }
  for (int i = kk + threadIdx.x; i < k; i += blockDim.x) dst[i] = -1;
  if (threadIdx.x == 0) out_n[row] = kk;
}

// Attention of each row over its selected keys: grid (rows, Hkv, ns), 128 threads,
// G query heads per KV head. Keys are processed in chunks of 128 (one per
// thread for the scores, one dim per thread for P.V). With ns > 1 (few rows, as in
// decode, where rows x Hkv CTAs would leave most SMs idle) split z takes an equal
// share of whole chunks and writes its unnormalised output with its running max and
// sum (log2 domain) to part[((row Hq + h) ns + z) (D + 2)]; dsa_attn_merge_kernel
// combines the splits. With ns == 1 the CTA writes the output directly.
template <int D, int G>
__global__ void __launch_bounds__(128) dsa_attn_kernel(const __nv_bfloat16* __restrict__ q, int q_ld,
                                                       const __nv_bfloat16* __restrict__ kc,
                                                       const __nv_bfloat16* __restrict__ vc, int Hkv,
                                                       const int* __restrict__ bt, int max_blocks,
                                                       const int* __restrict__ row_seq, const int* __restrict__ sel,
                                                       int sel_ld, const int* __restrict__ sel_n,
                                                       __nv_bfloat16* __restrict__ out, int out_ld, float scale_log2,
                                                       int num_blocks, int ns, float* __restrict__ part) {
  constexpr int NV = D / 8;
  __shared__ float qs[G][D];
  __shared__ float ps[G][128];
  __shared__ int kblk[128];
  __shared__ float alpha_s[G], m_s[G], l_s[G];
  const int row = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
  const int n = sel_n[row];
  const int per = (((n + 127) >> 7) + ns - 1) / ns * 128;  // keys of one split, whole chunks
  const int c_begin = z * per, c_end = min(n, c_begin + per);
  const int* srow = sel + (size_t)row * sel_ld;
  const int* btr = bt + (size_t)row_seq[row] * max_blocks;
  for (int i = tid; i < G * D; i += 128)
    qs[i / D][i % D] = __bfloat162float(q[(size_t)row * q_ld + (size_t)(kvh * G + i / D) * D + i % D]) * scale_log2;
  if (tid < G) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = 0.f;
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  for (int c0 = c_begin; c0 < c_end; c0 += 128) {
    const int cn = min(128, c_end - c0);
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = -INFINITY;
    if (tid < cn) {
      const int key = srow[c0 + tid];
      int blk = btr[key >> 4];
      blk = (blk < 0 || blk >= num_blocks) ? 0 : blk;
      const size_t rowoff = (((size_t)blk * Hkv + kvh) * 16 + (key & 15)) * D;
      kblk[tid] = (int)(rowoff / D);
      const uint4* kr = reinterpret_cast<const uint4*>(kc + rowoff);
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll 4
      for (int v = 0; v < NV; ++v) {
        const uint4 u = kr[v];
        const float k8[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                             bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int j = 0; j < 8; ++j) s[g] += qs[g][v * 8 + j] * k8[j];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) ps[g][tid] = s[g];
    __syncthreads();
    for (int g = warp; g < G; g += 4) {
      float mx = -INFINITY;
      for (int j = lane; j < 128; j += 32) mx = fmaxf(mx, ps[g][j]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m_s[g], mx);
      float sum = 0.f;
      for (int j = lane; j < 128; j += 32) {
        const float p = exp2f(ps[g][j] - mn);
        ps[g][j] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float al = exp2f(m_s[g] - mn);
        alpha_s[g] = al;
        l_s[g] = l_s[g] * al + sum;
        m_s[g] = mn;
      }
    }
    __syncthreads();
    if (tid < D) {
#pragma unroll
      for (int g = 0; g < G; ++g) o[g] *= alpha_s[g];
      for (int j = 0; j < cn; ++j) {
        const float v = __bfloat162float(vc[(size_t)kblk[j] * D + tid]);
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] += ps[g][j] * v;
      }
    }
    __syncthreads();
  }
  if (ns > 1) {
    const int Hq = gridDim.y * G;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float* pp = part + (((size_t)row * Hq + kvh * G + g) * ns + z) * (D + 2);
      if (tid < D) pp[tid] = o[g];
      if (tid == 0) {
        pp[D] = m_s[g];
        pp[D + 1] = l_s[g];
      }
    }
    return;
  }
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float l = l_s[g];
      out[(size_t)row * out_ld + (size_t)(kvh * G + g) * D + tid] = __float2bfloat16_rn(l > 0.f ? o[g] / l : 0.f);
    }
  }
}

// Combines the ns splits of dsa_attn_kernel: grid (rows, Hq), D threads.
// out = sum_z o_z 2^(m_z - M) / sum_z l_z 2^(m_z - M), M = max_z m_z; rows with no
// selected key (every m_z = -inf) get zeros.
template <int D>
__global__ void __launch_bounds__(D) dsa_attn_merge_kernel(const float* __restrict__ part, int ns,
                                                           __nv_bfloat16* __restrict__ out, int out_ld) {
  const int row = blockIdx.x, h = blockIdx.y, Hq = gridDim.y, tid = threadIdx.x;
  const float* pp = part + ((size_t)row * Hq + h) * ns * (D + 2);
  float M = -INFINITY;
  for (int z = 0; z < ns; ++z) M = fmaxf(M, pp[(size_t)z * (D + 2) + D]);
  float num = 0.f, den = 0.f;
  if (M > -INFINITY) {
    for (int z = 0; z < ns; ++z) {
      const float* q = pp + (size_t)z * (D + 2);
      const float w = exp2f(q[D] - M);  // 0 for an empty split (m = -inf)
      num += w * q[tid];
      den += w * q[D + 1];
    }
  }
  out[(size_t)row * out_ld + (size_t)h * D + tid] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
}

}  // namespace om

void om_dsa_scores(torch::Tensor qi, torch::Tensor wi, int64_t H, torch::Tensor icache, torch::Tensor bt,
                   torch::Tensor row_seq, torch::Tensor row_ctx, torch::Tensor scores, torch::Tensor status) {
  const int rows = row_seq.numel();
  if (rows == 0) return;
  TORCH_CHECK(H >= 1 && H <= om::DSA_MAX_HEADS && icache.size(-1) == om::DSA_DIM && icache.is_contiguous(),
              "dsa_scores: 1..8 heads of dim 64");
  TORCH_CHECK(wi.scalar_type() == at::kFloat && scores.scalar_type() == at::kFloat && scores.stride(1) == 1,
              "dsa_scores: fp32 weights / scores");
  const int s_ld = scores.size(1);
  dim3 grid(rows, (s_ld + 255) / 256);
  om::dsa_scores_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qi.data_ptr()), qi.stride(0), wi.data_ptr<float>(), wi.stride(0), H,
      reinterpret_cast<const __nv_bfloat16*>(icache.data_ptr()), bt.data_ptr<int>(), bt.size(1),
      row_seq.data_ptr<int>(), row_ctx.data_ptr<int>(), scores.data_ptr<float>(), s_ld, icache.size(0),
      status.data_ptr<int>());
  OM_LAUNCH_CHECK();
}

// scores [rows, s_ld] view (row stride s_ld); g [rows * H, >= S] bf16 from the indexer GEMM.
void om_dsa_head_reduce(torch::Tensor g, int64_t S, torch::Tensor w, int64_t H, torch::Tensor row_ctx,
                        torch::Tensor scores) {
  const int rows = row_ctx.numel();
  if (rows == 0) return;
  TORCH_CHECK(H >= 1 && H <= om::DSA_MAX_HEADS, "dsa_head_reduce: 1..8 heads");
  TORCH_CHECK(g.scalar_type() == at::kBFloat16 && g.stride(1) == 1 && g.size(0) == rows * H && g.size(1) >= S &&
                  g.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(g.data_ptr()) & 15) == 0,
              "dsa_head_reduce: g bf16 [rows * H, >= S], 16-byte aligned rows");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.size(0) == rows && scores.scalar_type() == at::kFloat &&
                  scores.stride(1) == 1 && scores.stride(0) == scores.size(1) && scores.size(0) == rows &&
                  row_ctx.scalar_type() == at::kInt,
              "dsa_head_reduce: w fp32 [rows, H], scores fp32 [rows, s_ld], row_ctx int32");
  const int s_ld = scores.size(1);
  dim3 grid((s_ld + 1023) / 1024, rows);
  om::dsa_head_reduce_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), g.stride(0), (int)S, w.data_ptr<float>(), w.stride(0),
      (int)H, row_ctx.data_ptr<int>(), scores.data_ptr<float>(), scores.stride(0));
  OM_LAUNCH_CHECK();
}

void om_dsa_topk(torch::Tensor scores, torch::Tensor row_ctx, int64_t k, torch::Tensor out_idx,
                 torch::Tensor out_n) {
  const int rows = scores.size(0), s_ld = scores.size(1);
  if (rows == 0) return;
  const size_t smem = (size_t)s_ld * 4;
  TORCH_CHECK(smem <= 200 * 1024, "dsa_topk: at most 51200 keys per row");
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(om::dsa_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev] = true;
  }
  om::dsa_topk_kernel<<<rows, 1024, smem, at::cuda::getCurrentCUDAStream().stream()>>>(
      scores.data_ptr<float>(), s_ld, row_ctx.data_ptr<int>(), k, out_idx.data_ptr<int>(), out_n.data_ptr<int>());
  OM_LAUNCH_CHECK();
}

void om_dsa_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor bt,
                      torch::Tensor row_seq, torch::Tensor sel, torch::Tensor sel_n, torch::Tensor out, int64_t Hq,
                      double scale) {
  const int rows = row_seq.numel();
  if (rows == 0) return;
  const int Hkv = k_cache.size(1), D = k_cache.size(3), G = Hq / Hkv;
  TORCH_CHECK(D == 128, "dsa_attention: head_dim 128");
  // Split the selected keys over ns CTAs per (row, KV head) when rows x Hkv would not
  // fill two waves of the GPU's SMs; at most one split per 128-key chunk.
  int sms = 148;
  {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int chunks = std::max(1, (int)((sel.size(1) + 127) / 128));
  const int want = (2 * sms + rows * Hkv - 1) / (rows * Hkv);
  const int ns = std::max(1, std::min(chunks, want));
  torch::Tensor part;
  if (ns > 1) part = torch::empty({(long)rows * Hq * ns * (D + 2)}, q.options().dtype(at::kFloat));
  float* part_ptr = ns > 1 ? part.data_ptr<float>() : nullptr;
  dim3 grid(rows, Hkv, ns);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto args = std::make_tuple(reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (int)q.stride(0),
                              reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()),
                              reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()), Hkv, bt.data_ptr<int>(),
                              (int)bt.size(1), row_seq.data_ptr<int>(), sel.data_ptr<int>(), (int)sel.size(1),
                              sel_n.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                              (int)out.stride(0), (float)(scale * 1.4426950408889634), (int)k_cache.size(0), ns,
                              part_ptr);
#define OM_DSA_LAUNCH(GG)                                                                              \
  std::apply([&](auto... xs) { om::dsa_attn_kernel<128, GG><<<grid, 128, 0, st>>>(xs...); }, args); \
  break;
  switch (G) {
    case 1: OM_DSA_LAUNCH(1)
    case 2: OM_DSA_LAUNCH(2)
    case 4: OM_DSA_LAUNCH(4)
    case 5: OM_DSA_LAUNCH(5)
    case 8: OM_DSA_LAUNCH(8)
    default: TORCH_CHECK(false, "dsa_attention: unsupported GQA group ", G);
  }
#undef OM_DSA_LAUNCH
  OM_LAUNCH_CHECK();
  if (ns > 1) {
    om::dsa_attn_merge_kernel<128><<<dim3(rows, Hq), 128, 0, st>>>(
        part_ptr, ns, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)out.stride(0));
    OM_LAUNCH_CHECK();
  }
}
