// Multi-head latent attention (MLA) over a paged latent cache, absorbed form.
//
// Every cached token is one 576-wide bf16 row: the RMS-normed 512-wide KV latent
// c followed by the 64-wide rotated key part k_r shared by all heads. With the
// per-head up-projections absorbed into the query (q_lat = W_uk^T q_nope, 512 wide,
// followed by the rotated q_r, 64 wide) a head's score against token t is
//     s = (q_lat . c_t + q_r . kr_t) * scale
// and its output in latent space is o_lat = sum_t softmax(s)_t c_t (512 wide); the
// caller applies W_uv and the output projection. All heads read the same rows, so
// a key tile is loaded once per 64-head group and reused by every head of it.
//
// Split over the context: CTA (partition p, row r, head group hg) handles tokens
// [64 p, 64 p + 64) of row r for heads [64 hg, 64 hg + 64):
//   1. q of the group and the 64 latent rows into shared memory (rows padded to
//      289 words so that lanes reading consecutive tokens hit different banks);
//   2. scores: thread = (token, 16 heads), the token's key word loaded once per k
//      and reused for its 16 heads;
//   3. softmax per head over the partition (warp per head) -> m, l, p;
//   4. o_part[h][d] = sum_t p[h][t] c_t[d]: thread = two latent columns, the column
//      kept in registers for all 64 tokens and reused by the 64 heads.
// A merge kernel combines the partitions: o = sum_p e^{m_p - M} o_p / sum_p e^{m_p - M} l_p.
//
// Bounds: rows whose sequence index, context or block id is out of range record
// OM_ERR_BOUNDS in the status word and contribute nothing.
//
// Reference counterpart: openmini-server/src/hardware/kv_cache/mla/{attention,
// latent_cache,projection}.rs and the MLA path of model/inference/model.rs:962-1027,
// 2381-2712 (CPU ndarray loops there; the math is the same latent attention).
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

#include <cuda_bf16.h>

namespace om {

constexpr int MLA_LAT = 512, MLA_ROPE = 64, MLA_ROW = MLA_LAT + MLA_ROPE;  // 576
constexpr int MLA_W = MLA_ROW / 2;       // 288 bf16x2 words per row
constexpr int MLA_WP = MLA_W + 1;        // padded shared-memory row (words)
constexpr int MLA_T = 64;                // tokens per partition
constexpr int MLA_HG = 64;               // heads per CTA
constexpr int MLA_NT = 256;

struct MlaArgs {
  const __nv_bfloat16* q;      // [rows, H, 576]
  const __nv_bfloat16* cache;  // [num_blocks, 16, 576]
  const int* block_tables;     // [num_seqs, max_blocks]
  const int* row_seq;          // [rows]
  const int* row_ctx;          // [rows]
  float* ws_o;                 // [rows, NP, H, 512]
  float* ws_ml;                // [rows, NP, H, 2]
  __nv_bfloat16* out;          // [rows, H, 512]
  int rows, H, NP, max_blocks, num_blocks, num_seqs;
  float scale;
  int* status;
};

__device__ __forceinline__ float2 bf2f(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ int mla_ctx(const MlaArgs& a, int r, int& seq) {
  seq = a.row_seq[r];
  int ctx = a.row_ctx[r];
  if (seq < 0 || seq >= a.num_seqs || ctx < 0 || ctx > a.max_blocks * 16 || ctx > a.NP * MLA_T) {
    record_error(a.status, OM_ERR_BOUNDS);
    return 0;
  }
  return ctx;
}

__global__ void __launch_bounds__(MLA_NT) mla_partial_kernel(const __grid_constant__ MlaArgs a) {
  extern __shared__ __align__(16) uint32_t sm[];
  uint32_t* qs = sm;                               // [MLA_HG][MLA_WP]
  uint32_t* ks = qs + MLA_HG * MLA_WP;             // [MLA_T][MLA_WP]
  float* sc = reinterpret_cast<float*>(ks + MLA_T * MLA_WP);  // [MLA_HG][MLA_T]
  const int p = blockIdx.x, r = blockIdx.y, hg = blockIdx.z;
  const int h0 = hg * MLA_HG;
  const int nh = min(MLA_HG, a.H - h0);
  int seq;
  const int ctx = mla_ctx(a, r, seq);
  const int start = p * MLA_T;
  const int n = max(0, min(MLA_T, ctx - start));
  float* wo = a.ws_o + (((size_t)r * a.NP + p) * a.H + h0) * MLA_LAT;
  float* wml = a.ws_ml + (((size_t)r * a.NP + p) * a.H + h0) * 2;
  if (n == 0) {
    for (int h = threadIdx.x; h < nh; h += MLA_NT) {
      wml[2 * h] = -INFINITY;
      wml[2 * h + 1] = 0.f;
    }
    return;
  }
  // 1. query group and key tile into shared memory
  const uint32_t* qg = reinterpret_cast<const uint32_t*>(a.q + ((size_t)r * a.H + h0) * MLA_ROW);
  for (int i = threadIdx.x; i < nh * MLA_W; i += MLA_NT) {
    const int h = i / MLA_W, w = i - h * MLA_W;
    qs[h * MLA_WP + w] = qg[(size_t)h * MLA_W + w];
  }
  const int* bt = a.block_tables + (size_t)seq * a.max_blocks;
  for (int i = threadIdx.x; i < MLA_T * MLA_W; i += MLA_NT) {
    const int t = i / MLA_W, w = i - t * MLA_W;
    uint32_t v = 0;
    if (t < n) {
      const int tok = start + t;
      const int blk = bt[tok >> 4];
      if (blk >= 0 && blk < a.num_blocks)
        v = reinterpret_cast<const uint32_t*>(a.cache + ((size_t)blk * 16 + (tok & 15)) * MLA_ROW)[w];
      else if (w == 0)
        record_error(a.status, OM_ERR_BOUNDS);
    }
    ks[t * MLA_WP + w] = v;
  }
  __syncthreads();
  // 2. scores: thread = token t, heads hb, hb + 4, ..., hb + 60
  {
    const int t = threadIdx.x & (MLA_T - 1);
    const int hb = threadIdx.x / MLA_T;  // 0..3
    float acc[MLA_HG / 4];
#pragma unroll
    for (int j = 0; j < MLA_HG / 4; ++j) acc[j] = 0.f;
    const uint32_t* kr = ks + t * MLA_WP;
    for (int w = 0; w < MLA_W; ++w) {
      const float2 kv = bf2f(kr[w]);
#pragma unroll
      for (int j = 0; j < MLA_HG / 4; ++j) {
        const float2 qv = bf2f(qs[(hb + 4 * j) * MLA_WP + w]);
        acc[j] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, acc[j]));
      }
    }
#pragma unroll
    for (int j = 0; j < MLA_HG / 4; ++j) {
      const int h = hb + 4 * j;
      sc[h * MLA_T + t] = (t < n && h < nh) ? acc[j] * a.scale : -INFINITY;
    }
  }
  __syncthreads();
  // 3. softmax per head over the partition: warp w takes heads w, w + 8, ...
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int h = warp; h < nh; h += MLA_NT / 32) {
      float* s = sc + h * MLA_T;
      const float x0 = s[lane], x1 = s[lane + 32];
      float m = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float e0 = __expf(x0 - m), e1 = __expf(x1 - m);
      float l = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      s[lane] = e0;
      s[lane + 32] = e1;
      if (lane == 0) {
        wml[2 * h] = m;
        wml[2 * h + 1] = l;
      }
    }
  }
  __syncthreads();
  // 4. o_part: thread = latent word w (columns 2w, 2w + 1), 256 words = 512 columns
  {
    const int w = threadIdx.x;
    float2 col[MLA_T];
#pragma unroll
    for (int t = 0; t < MLA_T; ++t) col[t] = bf2f(ks[t * MLA_WP + w]);
    for (int h = 0; h < nh; ++h) {
      const float* s = sc + h * MLA_T;
      float ox = 0.f, oy = 0.f;
#pragma unroll
      for (int t = 0; t < MLA_T; ++t) {
        ox = fmaf(s[t], col[t].x, ox);
        oy = fmaf(s[t], col[t].y, oy);
      }
      reinterpret_cast<float2*>(wo + (size_t)h * MLA_LAT)[w] = make_float2(ox, oy);
    }
  }
}

__global__ void __launch_bounds__(128) mla_merge_kernel(const __grid_constant__ MlaArgs a) {
  const int r = blockIdx.x, h = blockIdx.y;
  int seq;
  const int ctx = mla_ctx(a, r, seq);
  const int np = min(a.NP, (ctx + MLA_T - 1) / MLA_T);
  const float* ml = a.ws_ml + ((size_t)r * a.NP * a.H + h) * 2;
  float M = -INFINITY;
  for (int p = 0; p < np; ++p) M = fmaxf(M, ml[(size_t)p * a.H * 2]);
  float L = 0.f;
  for (int p = 0; p < np; ++p) L += __expf(ml[(size_t)p * a.H * 2] - M) * ml[(size_t)p * a.H * 2 + 1];
  const float inv = L > 0.f ? 1.f / L : 0.f;
  __nv_bfloat16* o = a.out + ((size_t)r * a.H + h) * MLA_LAT;
  for (int d = threadIdx.x; d < MLA_LAT; d += 128) {
    float acc = 0.f;
    for (int p = 0; p < np; ++p) {
      const float wgt = __expf(ml[(size_t)p * a.H * 2] - M);
      acc += wgt * a.ws_o[(((size_t)r * a.NP + p) * a.H + h) * MLA_LAT + d];
    }
    o[d] = __float2bfloat16_rn(acc * inv);
  }
}

}  // namespace om

int64_t om_mla_workspace(int64_t rows, int64_t H, int64_t max_ctx) {
  const int64_t np = (std::max<int64_t>(max_ctx, 1) + om::MLA_T - 1) / om::MLA_T;
  return rows * np * H * (om::MLA_LAT + 2);
}

// q [rows, H, 576] bf16 (absorbed latent query | rotated rope query), cache
// [num_blocks, 16, 576] bf16, out [rows, H, 512] bf16; ws fp32 of om_mla_workspace floats.
void om_mla_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables, torch::Tensor row_seq,
                   torch::Tensor row_ctx, torch::Tensor out, torch::Tensor ws, int64_t max_ctx, double scale,
                   torch::Tensor status) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 &&
                  q.size(2) == om::MLA_ROW, "mla: q must be contiguous bf16 [rows, H, 576]");
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.is_contiguous() && cache.dim() == 3 &&
                  cache.size(1) == 16 && cache.size(2) == om::MLA_ROW, "mla: cache must be bf16 [blocks, 16, 576]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == q.size(0) &&
                  out.size(1) == q.size(1) && out.size(2) == om::MLA_LAT, "mla: out must be bf16 [rows, H, 512]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous() && block_tables.dim() == 2,
              "mla: block_tables int32 [seqs, max_blocks]");
  TORCH_CHECK(row_seq.scalar_type() == at::kInt && row_ctx.scalar_type() == at::kInt &&
                  row_seq.numel() == q.size(0) && row_ctx.numel() == q.size(0), "mla: row_seq / row_ctx int32 [rows]");
  const int rows = q.size(0), H = q.size(1);
  if (rows == 0) return;
  const int64_t need = om_mla_workspace(rows, H, max_ctx);
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.is_contiguous() && ws.numel() >= need, "mla: workspace too small");
  om::MlaArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.cache = reinterpret_cast<const __nv_bfloat16*>(cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.row_seq = row_seq.data_ptr<int>();
  a.row_ctx = row_ctx.data_ptr<int>();
  a.rows = rows;
  a.H = H;
  a.NP = (int)((std::max<int64_t>(max_ctx, 1) + om::MLA_T - 1) / om::MLA_T);
  a.ws_o = ws.data_ptr<float>();
  a.ws_ml = a.ws_o + (size_t)rows * a.NP * H * om::MLA_LAT;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.max_blocks = block_tables.size(1);
  a.num_blocks = cache.size(0);
  a.num_seqs = block_tables.size(0);
  a.scale = (float)scale;
  a.status = status.data_ptr<int>();
  const size_t smem = (size_t)(om::MLA_HG + om::MLA_T) * om::MLA_WP * 4 + (size_t)om::MLA_HG * om::MLA_T * 4;
  static bool attr_set[64] = {false};
  int dev;
  OM_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(om::mla_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set[dev] = true;
  }
  auto st = at::cuda::getCurrentCUDAStream().stream();
  dim3 grid(a.NP, rows, (H + om::MLA_HG - 1) / om::MLA_HG);
  om::mla_partial_kernel<<<grid, om::MLA_NT, smem, st>>>(a);
  OM_LAUNCH_CHECK();
  om::mla_merge_kernel<<<dim3(rows, H), 128, 0, st>>>(a);
  OM_LAUNCH_CHECK();
}
