// Weight-only-quantised GEMM on the 5th-generation tensor cores:
//
//   Y = X @ dequant(Wq)^T,  X bf16 [M, K],  Wq 4-bit block-32 (Q4) or INT8 per-row (I8)
//
// The dequantisation is fused into the mainloop: the packed weight tile
// (128 rows x 64 k) is brought into shared memory in its compact form by one
// bulk copy (the device weight format stores every tile contiguously:
// [N/128][K/64][tile], tile = 128 rows x 32 B nibbles + 2 x 128 bf16 scales for
// Q4, 128 rows x 64 B for INT8, so the weight stream is strictly sequential),
// dequant warps expand it into the bf16 operand tile in exactly the
// 128-byte-swizzled K-major layout that tcgen05.mma reads, and the MMA issuer
// consumes it. HBM therefore carries 0.56 (Q4) or 1 (I8) byte per weight
// instead of 2.
//
// Three independent shared-memory rings keep the weight stream deep:
//   raw ring  packed weight tiles (+ Q4 scales), up to 24 slots, filled by the
//             weight producer, emptied once all dequant warps have read them
//   x ring    activation tiles (128-byte swizzle), filled by the activation
//             producer, emptied by the MMA
//   w ring    bf16 operand tiles, written by the dequant warps, emptied by the MMA
// so an activation reload never waits behind a weight slot and ~80-110 KB of
// packed weights stay in flight per SM.
//
// Roles (512 threads, one CTA per SM):
//   warp 0       TMA producer of the packed weights
//   warp 3       TMA producer of the activations
//   warp 1       MMA issuer (one elected lane), 2 TMEM accumulators
//   warp 2       TMEM allocation
//   warps 4..7   epilogue (shared with the bf16 kernel)
//   warps 8..15  dequant warps; all eight expand every tile together (16 rows
//                each, one 32-value half row per lane), so the latency from a raw
//                tile landing to its bf16 operand being ready is one eighth of a
//                tile's work and a 4-deep operand ring covers the MMA round trip.
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
  static constexpr int W_BYTES = 128 * BK * 2;  // bf16 operand tile
  static constexpr int X_BYTES = BX * BK * 2;   // activation tile
  static constexpr int RAW_Q = QT == WQ_Q4 ? 128 * 32 : 128 * 64;
  static constexpr int RAW_S = QT == WQ_Q4 ? 2 * 128 * 2 : 0;
  static constexpr int RAW_BYTES = RAW_Q + RAW_S;  // multiple of 16
  static constexpr int NDQ = 8;                   // dequant warps, 16 rows of every tile each
  static constexpr int WD = 4;                    // bf16 operand ring
  static constexpr int XD_ = (48 * 1024) / X_BYTES;
  static constexpr int XD = XD_ > 8 ? 8 : (XD_ < 2 ? 2 : XD_);
  static constexpr int RAW_AVAIL = 208 * 1024 - WD * W_BYTES - XD * X_BYTES;
  static constexpr int RD = RAW_AVAIL / RAW_BYTES > 24 ? 24 : RAW_AVAIL / RAW_BYTES;
  static_assert(RD >= 4, "raw ring too shallow");
  static constexpr int X_OFF = WD * W_BYTES;
  static constexpr int RAW_OFF = X_OFF + XD * X_BYTES;
  static constexpr int BAR_OFF = ((RAW_OFF + RD * RAW_BYTES + 15) / 16) * 16;
  static constexpr int SMEM_BYTES = BAR_OFF + (2 * WD + 2 * XD + 2 * RD + 4) * 8 + 16 + 1024;
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
    gemm_wq_tc_kernel(const __grid_constant__ CUtensorMap tmX, const GemmArgs g) {
  using C = WqCfg<BX, QT>;
  constexpr int BN_MMA = SWAP ? BX : 128;
  constexpr int TMEM_COLS = 2 * BN_MMA < 32 ? 32 : 2 * BN_MMA;
  constexpr int WD = C::WD, XD = C::XD, RD = C::RD, NDQ = C::NDQ;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wbuf = smem;
  uint8_t* xbuf = smem + C::X_OFF;
  uint8_t* rawbuf = smem + C::RAW_OFF;
  uint64_t* w_ready = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* w_empty = w_ready + WD;
  uint64_t* x_full = w_empty + WD;
  uint64_t* x_empty = x_full + XD;
  uint64_t* raw_full = x_empty + XD;
  uint64_t* raw_empty = raw_full + RD;
  uint64_t* tfull = raw_empty + RD;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = g.tiles_r * g.tiles_c * g.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WD; ++s) {
      mbar_init(&w_ready[s], NDQ);
      mbar_init(&w_empty[s], 1);
    }
    for (int s = 0; s < XD; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < RD; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], NDQ);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
  }
  if (warp == 2) tmem_alloc(tmem_slot, TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ producers
    if (elect_one()) {
      const bool wq = warp == 0;
      const int depth = wq ? RD : XD;
      uint64_t* fullb = wq ? raw_full : x_full;
      uint64_t* emptyb = wq ? raw_empty : x_empty;
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
          const int s = it % depth;
          const uint32_t ph = (it / depth) & 1;
          if (!mbar_wait(&emptyb[s], ph ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          if (wq) {
            uint8_t* raw = rawbuf + s * C::RAW_BYTES;
            mbar_arrive_expect_tx(&fullb[s], C::RAW_BYTES);
            // one contiguous bulk copy per pre-tiled weight block (sequential DRAM stream)
            bulk_load(raw, g.wtiles + ((size_t)wt * g.num_kb + kb) * C::RAW_BYTES, C::RAW_BYTES, &fullb[s]);
          } else {
            mbar_arrive_expect_tx(&fullb[s], C::X_BYTES);
            tma_load_2d(xbuf + s * C::X_BYTES, &tmX, &fullb[s], kb * 64, xt * BX);
          }
        }
      }
      if (!ok) {
        for (int j = max(0, it - depth); j < it; ++j) mbar_wait(&fullb[j % depth], (j / depth) & 1, nullptr, 0);
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
          const int xs = it % XD, ws = it % WD;
          if (!mbar_wait(&x_full[xs], (it / XD) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          if (!mbar_wait(&w_ready[ws], (it / WD) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(wbuf + ws * C::W_BYTES);
          const uint32_t x_addr = smem_u32(xbuf + xs * C::X_BYTES);
          const uint32_t a_addr = SWAP ? w_addr : x_addr;
          const uint32_t b_addr = SWAP ? x_addr : w_addr;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            tc_mma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32, 1024), smem_desc_sw128(b_addr + k * 32, 1024),
                       IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&x_empty[xs]);
          tc_commit(&w_empty[ws]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequant
    // All NDQ warps expand every tile together: warp d owns rows [16d, 16d + 16),
    // lane -> (row 16d + lane / 2, half lane % 2 of the 64 k values).
    const int d = warp - 8;
    const int row = d * 16 + (lane >> 1);
    const int half = lane & 1;
    const uint32_t sw = row & 7;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      int tr, tc, sp;
      unit_coords(g, u, tr, tc, sp);
      const int kb0 = sp * g.kb_per_split;
      const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int r = it % RD, s = it % WD;
        if (!mbar_wait(&raw_full[r], (it / RD) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
        const uint8_t* raw = rawbuf + r * C::RAW_BYTES;
        uint4 p0, p1;
        uint32_t s2 = 0;
        if (QT == WQ_Q4) {
          // block `half` of the row: 16 bytes of nibbles (32 values) and its scale
          p0 = *reinterpret_cast<const uint4*>(raw + row * 32 + half * 16);
          s2 = (uint32_t)reinterpret_cast<const uint16_t*>(raw + C::RAW_Q)[half * 128 + row] * 0x10001u;
        } else {
          p0 = *reinterpret_cast<const uint4*>(raw + row * 64 + half * 32);
          p1 = *reinterpret_cast<const uint4*>(raw + row * 64 + half * 32 + 16);
        }
        if (!mbar_wait(&w_empty[s], ((it / WD) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        uint8_t* wrow = wbuf + s * C::W_BYTES + row * 128;
        const uint32_t c0 = 4 * half;
        if (QT == WQ_Q4) {
          *reinterpret_cast<uint4*>(wrow + (((c0 + 0) ^ sw) << 4)) = q4_chunk(p0.x, p0.y, 0, s2);
          *reinterpret_cast<uint4*>(wrow + (((c0 + 1) ^ sw) << 4)) = q4_chunk(p0.z, p0.w, 0, s2);
          *reinterpret_cast<uint4*>(wrow + (((c0 + 2) ^ sw) << 4)) = q4_chunk(p0.x, p0.y, 4, s2);
          *reinterpret_cast<uint4*>(wrow + (((c0 + 3) ^ sw) << 4)) = q4_chunk(p0.z, p0.w, 4, s2);
        } else {
          *reinterpret_cast<uint4*>(wrow + (((c0 + 0) ^ sw) << 4)) = i8_chunk(p0.x, p0.y);
          *reinterpret_cast<uint4*>(wrow + (((c0 + 1) ^ sw) << 4)) = i8_chunk(p0.z, p0.w);
          *reinterpret_cast<uint4*>(wrow + (((c0 + 2) ^ sw) << 4)) = i8_chunk(p1.x, p1.y);
          *reinterpret_cast<uint4*>(wrow + (((c0 + 3) ^ sw) << 4)) = i8_chunk(p1.z, p1.w);
        }
        fence_proxy_async_smem();
        __syncwarp();
        // the raw slot is released only after every lane has read its part
        if (lane == 0) {
          mbar_arrive(&w_ready[s]);
          mbar_arrive(&raw_empty[r]);
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
