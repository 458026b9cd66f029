// Paged-KV decode attention on the 5th-generation tensor cores (head_dim 128,
// up to 16 query heads per KV head).
//
// Work item = (query row, KV head, partition of ATT_PART keys); a persistent
// CTA walks items and streams 128-key chunks of K and V from the paged cache
// with TMA (one 16-key paged block = two 16 x 64 boxes per tensor):
//
//   S^T[key, h] = K[key, :] . Q[h, :]        tcgen05.mma M=128 keys, N=16 heads, K=128 dims
//   online softmax over keys per head        4 warps, thread = key, TMEM -> registers
//   O^T[d, h]  += V^T[d, key] . P^T[key, h]   tcgen05.mma M=128 dims, N=16, K=128 keys
//
// The second product reads the V tile exactly as TMA stored it (keys as rows,
// dims contiguous): an MN-major A operand (LBO = distance between the two
// 64-dim halves, SBO = 8 key rows), so no transpose is needed. P is written by
// the softmax threads straight into the swizzled K-major B-operand layout.
// Running max / sum / output live in registers of the softmax warps (thread =
// key for S, thread = dim for O); partial results per partition are merged by
// attn_merge_kernel, as for the CUDA-core kernel in paged_attn.cu.
//
// Roles (256 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM
// owner, warps 4..7 softmax / output. Every wait is bounded.
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"
#include "attn_common.cuh"

namespace om {

namespace attn_tc {
constexpr int CH = 128;                 // keys per chunk
constexpr int HALF_BYTES = CH * 128;    // 128 keys x 64 dims bf16 = 16 KB
constexpr int KV_BYTES = 4 * HALF_BYTES;  // K (2 halves) + V (2 halves)
constexpr int STAGES = 3;
constexpr int Q_BYTES = 2 * 16 * 128;   // 16 heads x 128 dims
constexpr int P_BYTES = 2 * 16 * 128;   // 16 heads x 128 keys
constexpr int Q_OFF = STAGES * KV_BYTES;
constexpr int P_OFF = Q_OFF + Q_BYTES;
constexpr int BAR_OFF = P_OFF + P_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024 + 16 * 4 * 4 * 2;
}  // namespace attn_tc

struct AttnTcArgs {
  AttnArgs a;
  int G;        // query heads per KV head (<= 16)
  int items;    // rows * Hkv * NP
};

// Items are numbered partition-major: all (row, KV head) pairs of partition 0, then of
// partition 1, ... Partitions past a row's context are empty, and short rows only
// fill the low partitions, so with the partition varying fastest the round-robin
// deal gave some CTAs only empty items and others only full ones; partition-major
// numbering gives every CTA the same mix.
__device__ __forceinline__ void item_coords(const AttnTcArgs& t, int it, int& row, int& kvh, int& part) {
  const int per_part = t.items / t.a.NP;  // rows * Hkv
  part = it / per_part;
  const int r = it - part * per_part;
  kvh = r % t.a.Hkv;
  row = r / t.a.Hkv;
}

// NH: query heads handled per KV head in the softmax (G rounded up to 8 or 16; the
// MMA always computes 16 columns, the padded ones are never read).
template <int NH>
__global__ void __launch_bounds__(256, 1)
    paged_attn_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         const __grid_constant__ CUtensorMap tmQ, const AttnTcArgs t) {
  using namespace attn_tc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + Q_OFF;
  uint8_t* ps = smem + P_OFF;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* kv_empty = kv_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;   // [2]
  uint64_t* s_empty = s_full + 2;         // [2]
  uint64_t* q_full = s_empty + 2;
  uint64_t* q_empty = q_full + 1;
  uint64_t* p_full = q_empty + 1;
  uint64_t* p_empty = p_full + 1;
  uint64_t* o_full = p_empty + 1;
  uint64_t* o_empty = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 1);
  float* red = reinterpret_cast<float*>(smem + BAR_OFF + 256);  // [2][4 warps][16]

  const AttnArgs& a = t.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = a.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 128);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(p_full, 128);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 128);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, 64);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S[0]: cols 0-15, S[1]: 16-31, O: 32-47

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int cc = 0, ic = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < t.items && ok; it += gridDim.x) {
        int row, kvh, part;
        item_coords(t, it, row, kvh, part);
        int seq;
        const int ctx = checked_ctx(a, row, seq);
        const int start = part * ATT_PART;
        if (start >= ctx) continue;
        const int end = min(ctx, start + ATT_PART);
        const int* bt = a.block_tables + (size_t)seq * a.max_blocks;
        const int last_blk = (ctx - 1) >> 4;
        if (!mbar_wait(q_empty, (ic & 1) ^ 1, status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, Q_BYTES);
        tma_load_3d(qs, &tmQ, q_full, 0, kvh * t.G, row);
        tma_load_3d(qs + Q_BYTES / 2, &tmQ, q_full, 64, kvh * t.G, row);
        ++ic;
        for (int c0 = start; c0 < end; c0 += CH, ++cc) {
          const int s = cc % STAGES;
          if (!mbar_wait(&kv_empty[s], ((cc / STAGES) & 1) ^ 1, status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* st = smem + s * KV_BYTES;
          mbar_arrive_expect_tx(&kv_full[s], KV_BYTES);
#pragma unroll 1
          for (int b = 0; b < CH / 16; ++b) {
            // blocks past the context reuse the last valid block (finite data, masked in softmax)
            int blk = bt[min((c0 >> 4) + b, last_blk)];
            if (blk < 0 || blk >= a.num_blocks) {
              record_error(status, OM_ERR_BOUNDS);
              blk = 0;
            }
            const int y = (blk * a.Hkv + kvh) * 16;
            tma_load_2d(st + 0 * HALF_BYTES + b * 2048, &tmK, &kv_full[s], 0, y);
            tma_load_2d(st + 1 * HALF_BYTES + b * 2048, &tmK, &kv_full[s], 64, y);
            tma_load_2d(st + 2 * HALF_BYTES + b * 2048, &tmV, &kv_full[s], 0, y);
            tma_load_2d(st + 3 * HALF_BYTES + b * 2048, &tmV, &kv_full[s], 64, y);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 16);
      constexpr uint32_t IDESC_O = idesc_bf16_f32_amn(128, 16);
      const uint32_t q_addr = smem_u32(qs), p_addr = smem_u32(ps);
      int cc = 0, ic = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < t.items && ok; it += gridDim.x) {
        int row, kvh, part;
        item_coords(t, it, row, kvh, part);
        int seq;
        const int ctx = checked_ctx(a, row, seq);
        const int start = part * ATT_PART;
        if (start >= ctx) continue;
        const int nch = (min(ctx, start + ATT_PART) - start + CH - 1) / CH;
        if (!mbar_wait(q_full, ic & 1, status, OM_ERR_WAIT_FULL)) { ok = false; break; }
        ++ic;
        tc_fence_after();
        // S for chunk j is issued one chunk ahead of O for chunk j-1
        for (int j = 0; j <= nch && ok; ++j) {
          if (j < nch) {
            const int c = cc + j, s = c % STAGES, sb = c & 1;
            if (!mbar_wait(&kv_full[s], (c / STAGES) & 1, status, OM_ERR_WAIT_FULL)) { ok = false; break; }
            if (!mbar_wait(&s_empty[sb], ((c >> 1) & 1) ^ 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
            tc_fence_after();
            const uint32_t k_addr = smem_u32(smem + s * KV_BYTES);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t off = (k >> 2) * HALF_BYTES + (k & 3) * 32;
              const uint32_t qoff = (k >> 2) * (Q_BYTES / 2) + (k & 3) * 32;
              tc_mma_f16(tmem + sb * 16, smem_desc_sw128(k_addr + off, 1024), smem_desc_sw128(q_addr + qoff, 1024),
                         IDESC_S, k > 0 ? 1u : 0u);
            }
            tc_commit(&s_full[sb]);
            if (j == nch - 1) tc_commit(q_empty);
          }
          if (j > 0) {
            const int c = cc + j - 1, s = c % STAGES;
            if (!mbar_wait(p_full, c & 1, status, OM_ERR_WAIT_FULL)) { ok = false; break; }
            if (!mbar_wait(o_empty, (c & 1) ^ 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(smem + s * KV_BYTES + 2 * HALF_BYTES);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              // 16 keys per step: two 8-row swizzle atoms of V, 32 bytes of P
              const uint32_t poff = (k >> 2) * (P_BYTES / 2) + (k & 3) * 32;
              tc_mma_f16(tmem + 32, smem_desc_sw128_mn(v_addr + k * 2048, HALF_BYTES, 1024),
                         smem_desc_sw128(p_addr + poff, 1024), IDESC_O, k > 0 ? 1u : 0u);
            }
            tc_commit(o_full);
            tc_commit(p_empty);
            tc_commit(&kv_empty[s]);
          }
        }
        cc += nch;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax / output
    const int tid = threadIdx.x - 128;  // key within chunk (S) and dim (O)
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float* red_max = red;
    float* red_sum = red + 64;
    int cc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < t.items && ok; it += gridDim.x) {
      int row, kvh, part;
      item_coords(t, it, row, kvh, part);
      int seq;
        const int ctx = checked_ctx(a, row, seq);
      const int start = part * ATT_PART;
      if (start >= ctx) continue;
      const int end = min(ctx, start + ATT_PART);
      float m[16], l[16], acc[16];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
        acc[h] = 0.f;
      }
      for (int c0 = start; c0 < end; c0 += CH, ++cc) {
        const int sb = cc & 1;
        if (!mbar_wait(&s_full[sb], (cc >> 1) & 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[16];
        tmem_ld_32x32b_x16(tmem + lane_base + sb * 16, sr);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_empty[sb]);
        const bool valid = c0 + tid < end;
        float p[16], alpha[16];
#pragma unroll
        for (int h = 0; h < NH; ++h) p[h] = valid ? __uint_as_float(sr[h]) * a.scale_log2 : -INFINITY;
        // chunk max per head over the 128 keys
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          float v = p[h];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == 0) red_max[q * 16 + h] = v;
        }
        named_bar_sync(1, 128);
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const float cm = fmaxf(fmaxf(red_max[h], red_max[16 + h]), fmaxf(red_max[32 + h], red_max[48 + h]));
          const float mn = fmaxf(m[h], cm);
          alpha[h] = exp2f(m[h] - mn);  // 0 when m was -inf
          m[h] = mn;
          p[h] = valid ? exp2f(p[h] - mn) : 0.f;
        }
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          float v = p[h];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0) red_sum[q * 16 + h] = v;
        }
        // P^T -> smem (B operand, K-major: 16 head rows x 128 keys, two 64-key halves)
        if (!mbar_wait(p_empty, (cc & 1) ^ 1, status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        {
          uint8_t* ph = ps + (tid >> 6) * (P_BYTES / 2);
          const int kk = tid & 63;
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            const float v = h < t.G ? p[h] : 0.f;
            *reinterpret_cast<__nv_bfloat16*>(ph + h * 128 + ((((kk >> 3) ^ (h & 7))) << 4) + (kk & 7) * 2) =
                __float2bfloat16_rn(v);
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
#pragma unroll
        for (int h = 0; h < NH; ++h)
          l[h] = l[h] * alpha[h] + (red_sum[h] + red_sum[16 + h] + red_sum[32 + h] + red_sum[48 + h]);
        mbar_arrive(p_full);
        // O chunk: thread = output dim
        if (!mbar_wait(o_full, cc & 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
        tc_fence_after();
        uint32_t orr[16];
        tmem_ld_32x32b_x16(tmem + lane_base + 32, orr);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(o_empty);
        // the P ordering barrier above also keeps red_* stable until everyone read them
#pragma unroll
        for (int h = 0; h < NH; ++h) acc[h] = acc[h] * alpha[h] + __uint_as_float(orr[h]);
      }
      if (!ok) break;
      const size_t pbase = ((size_t)row * a.Hq + (size_t)kvh * t.G) * a.NP + part;
      for (int h = 0; h < t.G; ++h) a.part_o[(pbase + (size_t)h * a.NP) * 128 + tid] = acc[h];
      if (tid < t.G) {
        float mm = 0.f, ll = 0.f;
#pragma unroll
        for (int h = 0; h < NH; ++h)
          if (h == tid) { mm = m[h]; ll = l[h]; }
        a.part_ml[(pbase + (size_t)tid * a.NP) * 2 + 0] = mm;
        a.part_ml[(pbase + (size_t)tid * a.NP) * 2 + 1] = ll;
      }
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

}  // namespace om

// q [rows, >= Hq*128] (row stride q_ld), caches [blocks, Hkv, 16, 128]; same
// workspace contract as paged_attention (rows * Hq * NP * (128 + 2) floats).
void om_paged_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                           torch::Tensor row_seq, torch::Tensor row_ctx, torch::Tensor out, torch::Tensor workspace,
                           int64_t Hq, int64_t max_ctx, double scale, torch::Tensor status) {
  using namespace om::attn_tc;
  const int rows = row_seq.numel();
  if (rows == 0) return;
  const int Hkv = k_cache.size(1), D = k_cache.size(3);
  TORCH_CHECK(D == 128, "paged_attention_tc: head_dim must be 128");
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "paged_attention_tc: at most 16 query heads per KV head");
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1 && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "paged_attention_tc: layouts");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "block tables int32");
  om::AttnTcArgs t;
  om::AttnArgs& a = t.a;
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
              "paged_attention_tc: workspace too small");
  a.part_o = workspace.data_ptr<float>();
  a.part_ml = a.part_o + (size_t)rows * Hq * a.NP * D;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.num_blocks = k_cache.size(0);
  a.status = status.data_ptr<int>();
  t.G = Hq / Hkv;
  t.items = rows * Hkv * a.NP;
  const uint64_t cache_rows = (uint64_t)k_cache.size(0) * Hkv * 16;
  CUtensorMap tk = om::make_tmap_2d(a.kc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, cache_rows, 128, 64, 16,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = om::make_tmap_2d(a.vc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, cache_rows, 128, 64, 16,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tq = om::make_tmap_3d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, Hq, rows, 128, a.q_ld, 64, 16, 1,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(om::paged_attn_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    OM_CUDA_CHECK(cudaFuncSetAttribute(om::paged_attn_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    attr_set[dev] = true;
  }
  const int grid = std::min(t.items, om::num_sms());
  if (t.G <= 8)
    om::paged_attn_tc_kernel<8><<<grid, 256, SMEM_BYTES, st>>>(tk, tv, tq, t);
  else
    om::paged_attn_tc_kernel<16><<<grid, 256, SMEM_BYTES, st>>>(tk, tv, tq, t);
  OM_LAUNCH_CHECK();
  om::attn_merge_kernel<128><<<dim3(rows, Hq), 128, 0, st>>>(a);
  OM_LAUNCH_CHECK();
}
