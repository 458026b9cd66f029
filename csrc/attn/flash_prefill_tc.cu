// Paged-KV FlashAttention prefill on the 5th-generation tensor cores
// (head_dim 128, causal, GQA).
//
// Work item = (query tile of <= 128 consecutive rows of one sequence, query
// head). The host passes the tiles (row_start, rows, seq, keys of the last row),
// sorted by key count so that the longest items start first; a persistent CTA
// walks items. Per 128-key chunk of the paged cache (eight 16-key blocks, each
// brought in by TMA as two 16 x 64 boxes per tensor):
//
//   S[q, key] = Q[q, :] . K[key, :]     tcgen05.mma M=128 rows, N=128 keys, K=128 dims -> TMEM
//   softmax                             4 warps, thread = query row, S row read from TMEM
//   O[q, d]  += P[q, key] . V[key, d]   tcgen05.mma M=128, N=128 dims, K=128 keys -> TMEM
//
// V is read exactly as TMA stored it (keys as rows, dims contiguous): an
// MN-major B operand. S is double-buffered in TMEM (columns 0-255) so the MMA of
// chunk j+1 runs while chunk j is being exponentiated; O lives in TMEM columns
// 256-383 for the whole item.
//
// Lazy rescaling: each row keeps the max m it last exponentiated against and
// only moves it (rescaling O and l) when a chunk's max exceeds it by more than
// 2^8; otherwise exponents stay <= 8 and P <= 256, which bf16 / fp32 hold
// exactly enough. The final O / l is unaffected by which m was used.
//
// Roles (256 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM
// owner, warps 4..7 softmax and output. Every wait is bounded.
//
// Reference counterpart: the CPU blockwise online-softmax attention of
// openmini-server/src/model/inference/flash_attention_3.rs:280-420 (block 128)
// and the scalar kernel kernels.cu:220 (openmini-server/src/kernel/cuda).
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

namespace fa_pf {
constexpr int HALF = 128 * 128;          // 128 rows x 64 bf16 = 16 KB (one SW128 operand half)
constexpr int Q_BYTES = 2 * HALF;        // 128 rows x 128 dims
constexpr int KV_BYTES = 4 * HALF;       // K halves + V halves of a 128-key chunk
constexpr int STAGES = 2;
constexpr int P_BYTES = 2 * HALF;        // 128 rows x 128 keys
constexpr int KV_OFF = Q_BYTES;
constexpr int P_OFF = KV_OFF + STAGES * KV_BYTES;
constexpr int BAR_OFF = P_OFF + 2 * P_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr float RESCALE_LOG2 = 8.f;
}  // namespace fa_pf

struct PrefillArgs {
  const int* tiles;        // [ntiles][4] (row_start, rows, seq, keys of the last row), 4-byte aligned
  const int* row_ctx;      // [T] keys visible to each row
  const int* block_tables; // [S, max_blocks]
  __nv_bfloat16* out;      // [T, out_ld]
  int out_ld;
  int max_blocks, num_blocks;
  int Hq, Hkv, G;
  int items;               // ntiles * Hq
  float scale_log2;
  float* lse;              // optional [T, Hq] natural-log sum of exp of the scaled scores (ring merges)
  int* status;
};

__device__ __forceinline__ int4 load_tile(const int* tiles, int i) {
  const int* p = tiles + 4 * i;  // the tile list may sit at any 4-byte offset of a staging buffer
  return make_int4(p[0], p[1], p[2], p[3]);
}

__global__ void __launch_bounds__(256, 1)
    flash_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const PrefillArgs a) {
  using namespace fa_pf;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ps = smem + P_OFF;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* kv_empty = kv_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;  // [2]
  uint64_t* s_empty = s_full + 2;        // [2]
  uint64_t* p_full = s_empty + 2;        // [2]
  uint64_t* p_empty = p_full + 2;        // [2] (committed after the PV MMA that read P)
  uint64_t* q_full = p_empty + 2;
  uint64_t* q_empty = q_full + 1;
  uint64_t* o_empty = q_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 1);

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
      mbar_init(&p_full[b], 128);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_empty, 128);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 2) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S[0]: cols 0-127, S[1]: 128-255, O: 256-383

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int cc = 0, ic = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x, ++ic) {
        const int4 tl = load_tile(a.tiles, it / a.Hq);
        const int h = it % a.Hq, kvh = h / a.G;
        const int nch = (tl.w + 127) >> 7;
        const int* bt = a.block_tables + (size_t)tl.z * a.max_blocks;
        const int last_blk = (tl.w - 1) >> 4;
        if (!mbar_wait(q_empty, (ic & 1) ^ 1, status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, Q_BYTES);
        tma_load_2d(qs, &tmQ, q_full, h * 128, tl.x);
        tma_load_2d(qs + HALF, &tmQ, q_full, h * 128 + 64, tl.x);
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % STAGES;
          if (!mbar_wait(&kv_empty[s], ((cc / STAGES) & 1) ^ 1, status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* st = smem + KV_OFF + s * KV_BYTES;
          mbar_arrive_expect_tx(&kv_full[s], KV_BYTES);
#pragma unroll 1
          for (int b = 0; b < 8; ++b) {
            // blocks past the context reuse the last valid block (finite data, masked in softmax)
            int blk = bt[min(j * 8 + b, last_blk)];
            if (blk < 0 || blk >= a.num_blocks) {
              record_error(status, OM_ERR_BOUNDS);
              blk = 0;
            }
            const int y = (blk * a.Hkv + kvh) * 16;
            tma_load_2d(st + 0 * HALF + b * 2048, &tmK, &kv_full[s], 0, y);
            tma_load_2d(st + 1 * HALF + b * 2048, &tmK, &kv_full[s], 64, y);
            tma_load_2d(st + 2 * HALF + b * 2048, &tmV, &kv_full[s], 0, y);
            tma_load_2d(st + 3 * HALF + b * 2048, &tmV, &kv_full[s], 64, y);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128);
      constexpr uint32_t IDESC_O = idesc_bf16_f32_bmn(128, 128);
      const uint32_t q_addr = smem_u32(qs), p_addr = smem_u32(ps);
      int cc = 0, ic = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x, ++ic) {
        const int4 tl = load_tile(a.tiles, it / a.Hq);
        const int nch = (tl.w + 127) >> 7;
        if (!mbar_wait(q_full, ic & 1, status, OM_ERR_WAIT_FULL)) { ok = false; break; }
        tc_fence_after();
        // S of chunk j is issued one chunk ahead of O of chunk j-1
        for (int j = 0; j <= nch && ok; ++j) {
          if (j < nch) {
            const int c = cc + j, s = c % STAGES, sb = c & 1;
            if (!mbar_wait(&kv_full[s], (c / STAGES) & 1, status, OM_ERR_WAIT_FULL)) { ok = false; break; }
            if (!mbar_wait(&s_empty[sb], ((c >> 1) & 1) ^ 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
            tc_fence_after();
            const uint32_t k_addr = smem_u32(smem + KV_OFF + s * KV_BYTES);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t off = (k >> 2) * HALF + (k & 3) * 32;
              tc_mma_f16(tmem + sb * 128, smem_desc_sw128(q_addr + off, 1024), smem_desc_sw128(k_addr + off, 1024),
                         IDESC_S, k > 0 ? 1u : 0u);
            }
            tc_commit(&s_full[sb]);
            if (j == nch - 1) tc_commit(q_empty);
          }
          if (j > 0) {
            const int c = cc + j - 1, s = c % STAGES, pb = c & 1;
            if (!mbar_wait(&p_full[pb], (c >> 1) & 1, status, OM_ERR_WAIT_FULL)) { ok = false; break; }
            if (j == 1 && !mbar_wait(o_empty, (ic & 1) ^ 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(smem + KV_OFF + s * KV_BYTES + 2 * HALF);
            const uint32_t pa = p_addr + pb * P_BYTES;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              // 16 keys per step: 32 bytes of the P rows, two 8-key swizzle atoms of V
              tc_mma_f16(tmem + 256, smem_desc_sw128(pa + (k >> 2) * HALF + (k & 3) * 32, 1024),
                         smem_desc_sw128_mn(v_addr + k * 2048, HALF, 1024), IDESC_O, (j > 1 || k > 0) ? 1u : 0u);
            }
            tc_commit(&p_empty[pb]);
            tc_commit(&kv_empty[s]);
          }
        }
        cc += nch;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax / output
    const int t = threadIdx.x - 128;  // query row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    int cc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
      const int4 tl = load_tile(a.tiles, it / a.Hq);
      const int h = it % a.Hq;
      const int nch = (tl.w + 127) >> 7;
      const int my_ctx = t < tl.y ? a.row_ctx[tl.x + t] : 0;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nch; ++j) {
        const int c = cc + j, sb = c & 1;
        if (!mbar_wait(&s_full[sb], (c >> 1) & 1, status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
        tc_fence_after();
        uint32_t sv[128];
        tmem_ld_32x32b_x32(tmem + lane_base + sb * 128 + 0, *reinterpret_cast<uint32_t(*)[32]>(sv + 0));
        tmem_ld_32x32b_x32(tmem + lane_base + sb * 128 + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_ld_32x32b_x32(tmem + lane_base + sb * 128 + 64, *reinterpret_cast<uint32_t(*)[32]>(sv + 64));
        tmem_ld_32x32b_x32(tmem + lane_base + sb * 128 + 96, *reinterpret_cast<uint32_t(*)[32]>(sv + 96));
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_empty[sb]);
        const int lim = my_ctx - j * 128;  // valid columns of this chunk
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i < lim) mx = fmaxf(mx, __uint_as_float(sv[i]));
        const float m_cand = mx * a.scale_log2;
        // P[sb] is free once the PV MMA of chunk c-2 completed
        if (!mbar_wait(&p_empty[sb], ((c >> 1) & 1) ^ 1, status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        const bool need = m_cand > m_used + RESCALE_LOG2;
        // tcgen05.ld / st are warp-collective: a warp rescales together when any of its rows must
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O holds chunks < j: wait for the PV MMA of chunk c-1, then scale O and l
          const float m_new = fmaxf(m_used, m_cand);
          const float alpha = m_new == -INFINITY ? 1.f : fast_exp2(m_used - m_new);
          if (!mbar_wait(&p_empty[(c - 1) & 1], ((c - 1) >> 1) & 1, status, OM_ERR_WAIT_ACCUM)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int q = 0; q < 4; ++q) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tmem + lane_base + 256 + q * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x32(tmem + lane_base + 256 + q * 32, o);
          }
          tc_wait_st();
          l *= alpha;
          m_used = m_new;
        } else if (need) {
          m_used = m_cand;  // first chunk: O holds nothing yet
        }
        // P row -> smem (A operand, K-major SW128: two 64-key halves of 128-byte rows)
        float sum = 0.f;
        uint8_t* prow = ps + sb * P_BYTES + t * 128;
#pragma unroll
        for (int c8 = 0; c8 < 16; ++c8) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i0 = c8 * 8 + 2 * e;
            const float p0 = i0 < lim ? fast_exp2(__uint_as_float(sv[i0]) * a.scale_log2 - m_used) : 0.f;
            const float p1 = i0 + 1 < lim ? fast_exp2(__uint_as_float(sv[i0 + 1]) * a.scale_log2 - m_used) : 0.f;
            sum += p0 + p1;
            pk[e] = pack_bf16x2(p0, p1);
          }
          const int half = c8 >> 3, ch = c8 & 7;
          *reinterpret_cast<uint4*>(prow + half * HALF + ((ch ^ (t & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        l += sum;
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[sb]);
      }
      if (!ok) break;
      // O complete once the PV MMA of the last chunk committed
      const int last = cc + nch - 1;
      if (!mbar_wait(&p_empty[last & 1], (last >> 1) & 1, status, OM_ERR_WAIT_ACCUM)) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      if (a.lse != nullptr && t < tl.y)  // log-sum-exp of the row: (m_used + log2 l) in log2 units
        a.lse[(size_t)(tl.x + t) * a.Hq + h] = l > 0.f ? (m_used + log2f(l)) * 0.6931471805599453f : -INFINITY;
      __nv_bfloat16* orow = a.out + (size_t)(tl.x + t) * a.out_ld + h * 128;
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 256 + q * 32, o);
        tc_wait_ld();
        if (t < tl.y) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + q * 32 + v * 8) = w;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(o_empty);
      cc += nch;
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace om

// Causal prefill attention. q: [T, >= Hq*128] bf16 (row stride multiple of 8
// elements), caches [blocks, Hkv, 16, 128], tiles: int32 [ntiles, 4] on the
// device, rows of one tile belonging to one sequence and consecutive in q / out.
void om_flash_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor row_ctx, torch::Tensor tiles, torch::Tensor out, int64_t Hq, double scale,
                      torch::Tensor status, c10::optional<torch::Tensor> lse) {
  using namespace om::fa_pf;
  const int ntiles = tiles.size(0);
  if (ntiles == 0) return;
  const int Hkv = k_cache.size(1), D = k_cache.size(3);
  TORCH_CHECK(D == 128, "flash_prefill: head_dim must be 128");
  TORCH_CHECK(Hq % Hkv == 0, "flash_prefill: Hq % Hkv");
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1 && q.stride(0) % 8 == 0 && q.size(1) >= Hq * 128, "flash_prefill: q");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.stride(0) % 8 == 0, "flash_prefill: out");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "flash_prefill: caches");
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.is_contiguous() && tiles.size(1) == 4, "flash_prefill: tiles");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "block tables int32");
  om::PrefillArgs a;
  a.tiles = tiles.data_ptr<int>();
  a.row_ctx = row_ctx.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.max_blocks = block_tables.size(1);
  a.num_blocks = k_cache.size(0);
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.items = ntiles * Hq;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.status = status.data_ptr<int>();
  a.lse = nullptr;
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->is_contiguous() && lse->dim() == 2 &&
                    lse->size(0) >= q.size(0) && lse->size(1) == Hq,
                "flash_prefill: lse must be fp32 [T, Hq]");
    a.lse = lse->data_ptr<float>();
  }
  const uint64_t cache_rows = (uint64_t)k_cache.size(0) * Hkv * 16;
  CUtensorMap tk = om::make_tmap_2d(k_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, cache_rows, 128,
                                    64, 16, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = om::make_tmap_2d(v_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, cache_rows, 128,
                                    64, 16, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tq = om::make_tmap_2d(q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q.size(1), q.size(0),
                                    q.stride(0), 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    OM_CUDA_CHECK(cudaFuncSetAttribute(om::flash_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    attr_set[dev] = true;
  }
  const int grid = std::min(a.items, om::num_sms());
  om::flash_prefill_tc_kernel<<<grid, 256, SMEM_BYTES, st>>>(tq, tk, tv, a);
  OM_LAUNCH_CHECK();
}
