// Weight-only-quantised GEMM on the 5th-generation tensor cores:
//
//   Y = X @ dequant(Wq)^T,  X bf16 [M, K],  Wq 4-bit block-32 (Q4) or INT8 per-row (I8)
//
// The dequantisation is fused into the mainloop: the packed weight tile
// (128 rows x 64 k) is brought into shared memory by TMA in its compact form,
// eight dequant warps expand it into the bf16 operand tile in exactly the
// 128-byte-swizzled K-major layout that tcgen05.mma reads, and the MMA issuer
// consumes it. HBM therefore carries 0.56 (Q4) or 1 (I8) byte per weight
// instead of 2.
//
// Roles (512 threads, one CTA per SM):
//   warp 0       TMA producer: activation tile (swizzled) + packed weight tile + scales
//   warp 1       MMA issuer (one elected lane), 2 TMEM accumulators
//   warp 2       TMEM allocation
//   warps 4..7   epilogue (shared with the bf16 kernel)
//   warps 8..15  dequant: each warp expands whole stages (128 rows x 64 k), round robin
//
// SWAP = true (decode): A = weight tile (M = 128 weight rows), B = activations
// (N = BX tokens); the epilogue writes Y[token][row]. SWAP = false (prefill):
// A = activations (128 tokens), B = weight tile (N = 128 weight rows).
//
// Q4 element decode per pair: prmt the two source bytes into the two bf16
// halves, mask a nibble and OR the exponent of 128.0 (exact 128 + q), subtract
// 136 (exact), multiply by the block scale (one rounding).
// I8 element decode: fp32 magic-number conversion (exact), then packed
// conversion to bf16 (exact); the per-row scale is applied in the epilogue.
#pragma once
#include <cuda.h>
#include "gemm_common.cuh"

namespace om {

enum WQType : int { WQ_Q4 = 0, WQ_I8 = 1 };

template <int BX, int QT>
struct WqCfg {
  static constexpr int BK = 64;
  static constexpr int W_BYTES = 128 * BK * 2;   // bf16 operand tile
  static constexpr int X_BYTES = BX * BK * 2;
  static constexpr int RAW_Q = QT == WQ_Q4 ? 128 * 32 : 128 * 64;
  static constexpr int RAW_S = QT == WQ_Q4 ? 2 * 128 * 2 : 0;
  static constexpr int RAW_BYTES = RAW_Q + RAW_S;
  static constexpr int STAGE_BYTES = ((W_BYTES + X_BYTES + RAW_BYTES + 1023) / 1024) * 1024;
  static constexpr int STAGES_ = (200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_ > 8 ? 8 : STAGES_;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
};

__device__ __forceinline__ uint32_t q4_pair(uint32_t t, int shift, uint32_t s2) {
  uint32_t v = ((t >> shift) & 0x000F000Fu) | 0x43004300u;
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  const uint32_t off = 0x43084308u;  // bf16x2(136, 136)
  b = __hsub2(b, *reinterpret_cast<const __nv_bfloat162*>(&off));
  b = __hmul2(b, *reinterpret_cast<const __nv_bfloat162*>(&s2));
  return *reinterpret_cast<uint32_t*>(&b);
}

// 8 packed bytes (lo nibbles or hi nibbles) -> one 16-byte chunk of 8 bf16
__device__ __forceinline__ uint4 q4_chunk(uint32_t w0, uint32_t w1, int shift, uint32_t s2) {
  uint4 o;
  o.x = q4_pair(__byte_perm(w0, 0, 0x4140), shift, s2);
  o.y = q4_pair(__byte_perm(w0, 0, 0x4342), shift, s2);
  o.z = q4_pair(__byte_perm(w1, 0, 0x4140), shift, s2);
  o.w = q4_pair(__byte_perm(w1, 0, 0x4342), shift, s2);
  return o;
}

__device__ __forceinline__ float i8_at(uint32_t w, int byte) {
  const uint32_t u = ((w >> (8 * byte)) ^ 0x80u) & 0xFFu;
  return __uint_as_float(0x4B000000u | u) - 8388736.f;
}
__device__ __forceinline__ uint4 i8_chunk(uint32_t w0, uint32_t w1) {
  uint4 o;
  o.x = pack_bf16x2(i8_at(w0, 0), i8_at(w0, 1));
  o.y = pack_bf16x2(i8_at(w0, 2), i8_at(w0, 3));
  o.z = pack_bf16x2(i8_at(w1, 0), i8_at(w1, 1));
  o.w = pack_bf16x2(i8_at(w1, 2), i8_at(w1, 3));
  return o;
}

template <int BX, int QT, bool SWAP>
__global__ void __launch_bounds__(512, 1)
    gemm_wq_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmS, const GemmArgs g) {
  using C = WqCfg<BX, QT>;
  constexpr int BN_MMA = SWAP ? BX : 128;
  constexpr int TMEM_COLS = 2 * BN_MMA < 32 ? 32 : 2 * BN_MMA;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* wready = full + C::STAGES;
  uint64_t* empty = wready + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = g.tiles_r * g.tiles_c * g.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&wready[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmQ);
    if (QT == WQ_Q4) tma_prefetch_desc(&tmS);
  }
  if (warp == 2) tmem_alloc(tmem_slot, TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int tr, tc, sp;
        unit_coords(g, u, tr, tc, sp);
        const int wt = SWAP ? tr : tc;  // weight tile (128 rows)
        const int xt = SWAP ? tc : tr;  // activation tile (BX rows)
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE_BYTES;
          uint8_t* xs = st + C::W_BYTES;
          uint8_t* raw = xs + C::X_BYTES;
          mbar_arrive_expect_tx(&full[s], C::X_BYTES + C::RAW_BYTES);
          tma_load_2d(xs, &tmX, &full[s], kb * 64, xt * BX);
          if (QT == WQ_Q4) {
            tma_load_2d(raw, &tmQ, &full[s], kb * 32, wt * 128);
            tma_load_2d(raw + C::RAW_Q, &tmS, &full[s], wt * 128, kb * 2);
          } else {
            tma_load_2d(raw, &tmQ, &full[s], kb * 64, wt * 128);
          }
        }
      }
      if (!ok) {
        for (int j = max(0, it - C::STAGES); j < it; ++j)
          mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BN_MMA);
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++local) {
        int tr, tc, sp;
        unit_coords(g, u, tr, tc, sp);
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, g.status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN_MMA;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          if (!mbar_wait(&wready[s], ph, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t x_addr = w_addr + C::W_BYTES;
          const uint32_t a_addr = SWAP ? w_addr : x_addr;
          const uint32_t b_addr = SWAP ? x_addr : w_addr;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            tc_mma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32, 1024), smem_desc_sw128(b_addr + k * 32, 1024),
                       IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequant
    // Warp d handles every NDQ-th stage iteration on its own (one fence per
    // stage per warp), so up to NDQ stages are expanded concurrently. NDQ never
    // exceeds the ring depth, so two warps never wait on the same barrier phase.
    constexpr int NDQ = C::STAGES < 8 ? C::STAGES : 8;
    const int d = warp - 8;
    if (d < NDQ) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int tr, tc, sp;
        unit_coords(g, u, tr, tc, sp);
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          if (it % NDQ != d) continue;
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE_BYTES;
          const uint8_t* raw = st + C::W_BYTES + C::X_BYTES;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int row = lane + 32 * j;
            uint8_t* wrow = st + row * 128;
            const uint32_t sw = row & 7;
            if (QT == WQ_Q4) {
              const uint4 p0 = *reinterpret_cast<const uint4*>(raw + row * 32);
              const uint4 p1 = *reinterpret_cast<const uint4*>(raw + row * 32 + 16);
              const uint16_t* sc = reinterpret_cast<const uint16_t*>(raw + C::RAW_Q);
              const uint32_t s0 = (uint32_t)sc[row] * 0x10001u;
              const uint32_t s1 = (uint32_t)sc[128 + row] * 0x10001u;
              *reinterpret_cast<uint4*>(wrow + ((0 ^ sw) << 4)) = q4_chunk(p0.x, p0.y, 0, s0);
              *reinterpret_cast<uint4*>(wrow + ((1 ^ sw) << 4)) = q4_chunk(p0.z, p0.w, 0, s0);
              *reinterpret_cast<uint4*>(wrow + ((2 ^ sw) << 4)) = q4_chunk(p0.x, p0.y, 4, s0);
              *reinterpret_cast<uint4*>(wrow + ((3 ^ sw) << 4)) = q4_chunk(p0.z, p0.w, 4, s0);
              *reinterpret_cast<uint4*>(wrow + ((4 ^ sw) << 4)) = q4_chunk(p1.x, p1.y, 0, s1);
              *reinterpret_cast<uint4*>(wrow + ((5 ^ sw) << 4)) = q4_chunk(p1.z, p1.w, 0, s1);
              *reinterpret_cast<uint4*>(wrow + ((6 ^ sw) << 4)) = q4_chunk(p1.x, p1.y, 4, s1);
              *reinterpret_cast<uint4*>(wrow + ((7 ^ sw) << 4)) = q4_chunk(p1.z, p1.w, 4, s1);
            } else {
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const uint4 p = *reinterpret_cast<const uint4*>(raw + row * 64 + h * 16);
                *reinterpret_cast<uint4*>(wrow + (((2 * h) ^ sw) << 4)) = i8_chunk(p.x, p.y);
                *reinterpret_cast<uint4*>(wrow + (((2 * h + 1) ^ sw) << 4)) = i8_chunk(p.z, p.w);
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&wready[s]);
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++local) {
      int tr, tc, sp;
      unit_coords(g, u, tr, tc, sp);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], aph, g.status, OM_ERR_WAIT_ACCUM)) break;
      tc_fence_after();
      const int r = tr * 128 + q * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN_MMA;
#pragma unroll 1
      for (int cc = 0; cc < BN_MMA / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + cc * 32, v);
        tc_wait_ld();
        epilogue_chunk(g, v, r, tc * BN_MMA + cc * 32, sp);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace om
