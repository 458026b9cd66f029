// Paged-KV attention over "query rows": every row t has its own query vector
// (all heads), a sequence (-> block table) and a count of visible keys. Decode
// is one row per sequence; causal prefill is one row per prompt token with
// ctx_len = position + 1, so one kernel serves both.
//
// Split-KV (flash-decoding): grid (rows, kv_heads, partitions of PART keys).
// Each CTA handles the G = Hq/Hkv query heads that share one KV head (GQA),
// keeps a running max / sum per head (online softmax in base 2), and writes an
// unnormalised partial; a second kernel merges the partitions. K/V are read
// once per (row, kv head): the G query heads reuse each K/V row from registers.
//
// Restates (math only) openmini-server/src/kernel/cuda/kernels.cu:220-285 and
// openmini-server/src/hardware/gpu/cuda.rs:497-547 (online-softmax attention),
// openmini-server/src/model/inference/model.rs:1468-1540 (causal GQA attention)
// and openmini-server/src/hardware/kv_cache/paged_cache.rs:110-435 (paged read).
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"
#include "attn_common.cuh"

namespace om {


template <int D, int G>
__global__ void __launch_bounds__(128) paged_attn_kernel(const AttnArgs a) {
  constexpr int NT = 128;
  constexpr int NV = D / 8;  // uint4 per K/V row
  __shared__ float qs[G][D];
  __shared__ float ps[G][ATT_CHUNK];
  __shared__ float alpha_s[G];
  __shared__ float m_s[G], l_s[G];

  const int row = blockIdx.x, kvh = blockIdx.y, part = blockIdx.z;
  int seq;
  const int ctx = checked_ctx(a, row, seq);
  const int start = part * ATT_PART;
  const int tid = threadIdx.x;
  const size_t pbase = ((size_t)row * a.Hq + (size_t)kvh * G) * a.NP + part;
  if (start >= ctx) {
    // empty partition: contribute nothing to the merge
    if (tid < G) {
      a.part_ml[(pbase + (size_t)tid * a.NP) * 2 + 0] = -INFINITY;
      a.part_ml[(pbase + (size_t)tid * a.NP) * 2 + 1] = 0.f;
    }
    return;
  }
  const int end = min(ctx, start + ATT_PART);
  const int* bt = a.block_tables + (size_t)seq * a.max_blocks;

  for (int i = tid; i < G * D; i += NT) {
    const int g = i / D, d = i % D;
    qs[g][d] = __bfloat162float(a.q[(size_t)row * a.q_ld + (size_t)(kvh * G + g) * D + d]) * a.scale_log2;
  }
  if (tid < G) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = 0.f;
  __syncthreads();

  const int warp = tid >> 5, lane = tid & 31;
  for (int c0 = start; c0 < end; c0 += ATT_CHUNK) {
    const int n = min(ATT_CHUNK, end - c0);
    // ---- scores: thread tid owns key c0 + tid
    {
      float s[G];
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = -INFINITY;
      if (tid < n) {
        const int key = c0 + tid;
        int blk = bt[key >> 4];
        if (blk < 0 || blk >= a.num_blocks) {
          record_error(a.status, OM_ERR_BOUNDS);
          blk = 0;
        }
        const uint4* kr = reinterpret_cast<const uint4*>(a.kc + (((size_t)blk * a.Hkv + kvh) * 16 + (key & 15)) * D);
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll 4
        for (int v = 0; v < NV; ++v) {
          const uint4 u = kr[v];
          float k8[8];
          k8[0] = bf16lo(u.x); k8[1] = bf16hi(u.x); k8[2] = bf16lo(u.y); k8[3] = bf16hi(u.y);
          k8[4] = bf16lo(u.z); k8[5] = bf16hi(u.z); k8[6] = bf16lo(u.w); k8[7] = bf16hi(u.w);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float4 qa = *reinterpret_cast<const float4*>(&qs[g][v * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&qs[g][v * 8 + 4]);
            s[g] += qa.x * k8[0] + qa.y * k8[1] + qa.z * k8[2] + qa.w * k8[3] + qb.x * k8[4] + qb.y * k8[5] +
                    qb.z * k8[6] + qb.w * k8[7];
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) ps[g][tid] = s[g];
    }
    __syncthreads();
    // ---- online softmax update, one warp per head (round robin)
    for (int g = warp; g < G; g += NT / 32) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < ATT_CHUNK / 32; ++j) mx = fmaxf(mx, ps[g][lane + 32 * j]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = m_s[g];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < ATT_CHUNK / 32; ++j) {
        const float p = exp2f(ps[g][lane + 32 * j] - m_new);
        ps[g][lane + 32 * j] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float al = exp2f(m_old - m_new);
        alpha_s[g] = al;
        l_s[g] = l_s[g] * al + sum;
        m_s[g] = m_new;
      }
    }
    __syncthreads();
    // ---- PV: thread tid owns output dim tid (D=64 uses half the threads)
    if (tid < D) {
#pragma unroll
      for (int g = 0; g < G; ++g) o[g] *= alpha_s[g];
      int cur_blk = -1;
      const __nv_bfloat16* vb = nullptr;
#pragma unroll 4
      for (int j = 0; j < n; ++j) {
        const int key = c0 + j;
        const int bi = key >> 4;
        if (bi != cur_blk) {
          cur_blk = bi;
          int blk = bt[bi];
          if (blk < 0 || blk >= a.num_blocks) blk = 0;
          vb = a.vc + (((size_t)blk * a.Hkv + kvh) * 16) * D;
        }
        const float v = __bfloat162float(vb[(key & 15) * D + tid]);
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] += ps[g][j] * v;
      }
    }
    __syncthreads();
  }
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < G; ++g) a.part_o[(pbase + (size_t)g * a.NP) * D + tid] = o[g];
  }
  if (tid < G) {
    a.part_ml[(pbase + (size_t)tid * a.NP) * 2 + 0] = m_s[tid];
    a.part_ml[(pbase + (size_t)tid * a.NP) * 2 + 1] = l_s[tid];
  }
}


template <int D>
static void launch_d(const AttnArgs& a, int rows, int G, cudaStream_t st) {
  dim3 grid(rows, a.Hkv, a.NP);
  switch (G) {
    case 1: paged_attn_kernel<D, 1><<<grid, 128, 0, st>>>(a); break;
    case 2: paged_attn_kernel<D, 2><<<grid, 128, 0, st>>>(a); break;
    case 4: paged_attn_kernel<D, 4><<<grid, 128, 0, st>>>(a); break;
    case 5: paged_attn_kernel<D, 5><<<grid, 128, 0, st>>>(a); break;
    case 8: paged_attn_kernel<D, 8><<<grid, 128, 0, st>>>(a); break;
    case 16: paged_attn_kernel<D, 16><<<grid, 128, 0, st>>>(a); break;
    default: TORCH_CHECK(false, "paged_attention: unsupported GQA group ", G);
  }
  OM_LAUNCH_CHECK();
  attn_merge_kernel<D><<<dim3(rows, a.Hq), 128, 0, st>>>(a);
  OM_LAUNCH_CHECK();
}

}  // namespace om

// max_ctx bounds the number of partitions (fixed for CUDA-graph capture).
void om_paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                        torch::Tensor row_seq, torch::Tensor row_ctx, torch::Tensor out, torch::Tensor workspace,
                        int64_t Hq, int64_t max_ctx, double scale, torch::Tensor status) {
  const int rows = row_seq.numel();
  if (rows == 0) return;
  const int Hkv = k_cache.size(1), D = k_cache.size(3);
  TORCH_CHECK(Hq % Hkv == 0, "paged_attention: Hq % Hkv");
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "paged_attention: inner dims contiguous");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "block tables int32");
  om::AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_ld = q.stride(0);
  a.kc = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.vc = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = block_tables.size(1);
  a.num_seqs = block_tables.size(0);
  a.row_seq = row_seq.data_ptr<int>();
  a.row_ctx = row_ctx.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.NP = std::max<int64_t>(1, (max_ctx + om::ATT_PART - 1) / om::ATT_PART);
  const size_t need = (size_t)rows * Hq * a.NP * (D + 2);
  TORCH_CHECK(workspace.scalar_type() == at::kFloat && (size_t)workspace.numel() >= need,
              "paged_attention: workspace too small (need ", need, " floats)");
  a.part_o = workspace.data_ptr<float>();
  a.part_ml = a.part_o + (size_t)rows * Hq * a.NP * D;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.num_blocks = k_cache.size(0);
  a.status = status.data_ptr<int>();
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (D == 128)
    om::launch_d<128>(a, rows, Hq / Hkv, st);
  else if (D == 64)
    om::launch_d<64>(a, rows, Hq / Hkv, st);
  else
    TORCH_CHECK(false, "paged_attention: head_dim must be 64 or 128");
}

int64_t om_paged_attention_workspace(int64_t rows, int64_t Hq, int64_t D, int64_t max_ctx) {
  const int64_t np = std::max<int64_t>(1, (max_ctx + om::ATT_PART - 1) / om::ATT_PART);
  return rows * Hq * np * (D + 2);
}

// ============================================================================
// Allocation-free C entry point for paged attention.
//
// This entry point has no counterpart in the reference. It exists for callers
// that must not allocate device memory: code running inside a custom memory
// pool or allocator hook, plugins hosted by another runtime that owns all
// device memory, or real-time paths where a cudaMalloc could block or fail at
// the wrong moment. Such callers pass only their inputs and outputs; the
// split-KV partial results live in a fixed device array owned by this library.
//
// Limits and behaviour:
//   * The scratch array holds OM_NOALLOC_SCRATCH_FLOATS fp32 values (16 MiB).
//   * Rows whose sequence index or context exceeds the block table or max_ctx
//     set OM_ERR_BOUNDS (5) in *status and are clamped; the call still returns 0.
//     A call needs rows * Hq * ceil(max_ctx / 512) * (head_dim + 2) floats and
//     is rejected with OM_NOALLOC_TOO_LARGE if that exceeds the array.
//   * Every GPU that loads this library reserves the 16 MiB until the process
//     exits.
//   * The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress with that device current) and caches it; make that
//     first call before any stream capture.
//   * All calls share the one array, which keeps the previous call's contents.
//     Calls whose kernels overlap on the GPU (different streams, or several
//     host threads) race on it; serialise them. Nothing in it needs clearing:
//     every partial the merge kernel reads is written earlier in the same call.
//   * No cudaMalloc / cudaFree or allocating library routine is called.
// ============================================================================
#include <mutex>
#include "../../include/openmini_b200.h"

static __device__ __align__(256) float om_noalloc_scratch[OM_NOALLOC_SCRATCH_FLOATS];

static float* om_noalloc_scratch_ptr() {
  static std::mutex mu;
  static float* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, om_noalloc_scratch) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<float*>(p);
  }
  return ptrs[dev];
}

// Declared in include/openmini_b200.h (arguments and return codes documented there).
extern "C" int om_paged_attention_noalloc(const void* q, int q_ld, const void* k_cache, const void* v_cache,
                                          int num_blocks, int Hkv, int head_dim, const int* block_tables,
                                          int num_seqs, int max_blocks, const int* row_seq, const int* row_ctx,
                                          int rows, void* out, int out_ld, int Hq, int max_ctx, float scale,
                                          int* status, cudaStream_t stream) {
  if (rows <= 0) return OM_NOALLOC_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !row_seq || !row_ctx || !out) return OM_NOALLOC_BAD_ARGS;
  if (Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0 || (head_dim != 64 && head_dim != 128) || max_ctx <= 0 ||
      num_seqs <= 0 || max_blocks <= 0 || num_blocks <= 0)
    return OM_NOALLOC_BAD_ARGS;
  const int G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 5 && G != 8 && G != 16) return OM_NOALLOC_BAD_ARGS;
  // partitions in 64-bit, and the size check as a quotient so no product can wrap
  const int64_t np = ((int64_t)max_ctx + om::ATT_PART - 1) / om::ATT_PART;
  const uint64_t per_part = (uint64_t)rows * (uint64_t)Hq * (uint64_t)(head_dim + 2);
  if ((uint64_t)np > OM_NOALLOC_SCRATCH_FLOATS / per_part) return OM_NOALLOC_TOO_LARGE;
  float* scratch = om_noalloc_scratch_ptr();
  if (!scratch) return OM_NOALLOC_CUDA_ERROR;
  om::AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_ld = q_ld;
  a.kc = static_cast<const __nv_bfloat16*>(k_cache);
  a.vc = static_cast<const __nv_bfloat16*>(v_cache);
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.num_seqs = num_seqs;
  a.row_seq = row_seq;
  a.row_ctx = row_ctx;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_ld = out_ld;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.NP = (int)np;
  a.part_o = scratch;
  a.part_ml = scratch + (size_t)rows * Hq * np * head_dim;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.num_blocks = num_blocks;
  a.status = status;
  try {
    if (head_dim == 128)
      om::launch_d<128>(a, rows, G, stream);
    else
      om::launch_d<64>(a, rows, G, stream);
  } catch (...) {
    return OM_NOALLOC_CUDA_ERROR;
  }
  return OM_NOALLOC_OK;
}
