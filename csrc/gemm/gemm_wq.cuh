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
//   warps 8..15  dequant warps in NG = 4 groups of 2: group g expands the tiles
//                it = g (mod 4), so four tiles are expanded at once and every warp
//                does 64 rows of a tile per iteration (the fixed cost of one
//                iteration -- barrier waits, proxy fence, arrivals -- is paid
//                once per 4096 weights and hidden by the other groups). The
//                rings' depths are multiples of NG, so a slot is always
//                consumed by the same group and no waiter can run a full lap
//                ahead of a barrier phase.
// Weight copies are chunked: CH consecutive K blocks of a weight row-tile are
// contiguous in the device format and move as one bulk copy (18 KB for Q4), and
// the activations for the same CH K blocks as one 3-D TMA box, because every
// copy costs a fixed issue time on its thread and 4.6 KB copies capped one
// issuing thread near half of HBM bandwidth (measured on B200).
//
// SWAP = true (decode): A = weight tile (M = 128 weight rows), B = activations
// (N = BX tokens); the epilogue writes Y[token][row]. A work unit covers
// g.rgroup consecutive weight row-tiles (up to 256 / BX): every activation tile
// brought in by TMA feeds that many MMAs into as many TMEM accumulators, so the
// activation stream (which equals the packed weight stream in bytes at 32
// tokens) shrinks by that factor and the activation ring stops limiting the
// weight stream. SWAP = false (prefill):
// A = activations (128 tokens), B = weight tile (N = 128 weight rows).
//
// Q4 element decode per pair (q4_pair): mask two nibbles of one word and OR the
// exponent of 128.0 (exact 128 + q), subtract 136 (exact), multiply by the block
// scale (one rounding). I8 element decode (i8_pair): fp32 magic-number
// conversion (exact), then packed conversion to bf16 (exact); the per-row scale
// is applied in the epilogue. Decode with M <= 128 tokens uses the TMEM-operand
// kernel of gemm_wq_dec.cuh; this kernel serves larger M and prefill.
#pragma once
#include <cuda.h>
#include "gemm_common.cuh"

namespace om {

enum WQType : int { WQ_Q4 = 0, WQ_I8 = 1 };

template <int BX, int QT, bool SWAP>
struct WqCfg {
  static constexpr int BK = 64;
  static constexpr int W_BYTES = 128 * BK * 2;  // bf16 operand tile
  static constexpr int X_BYTES = BX * BK * 2;   // activation tile (one kb)
  static constexpr int RAW_Q = QT == WQ_Q4 ? 128 * 32 : 128 * 64;
  static constexpr int RAW_S = QT == WQ_Q4 ? 2 * 128 * 2 : 0;
  static constexpr int RAW_BYTES = RAW_Q + RAW_S;  // multiple of 16
  static constexpr int NDQ = 8;                   // dequant warps
  static constexpr int NG = 4;                    // dequant groups (tiles expanded concurrently)
  static constexpr int WPG = NDQ / NG;            // warps per tile
  static constexpr int RPW = 128 / WPG;           // rows of a tile per warp
  static constexpr int WD = 4;                    // bf16 operand ring (multiple of NG)
  // kb per chunk (g.chunk <= CHMAX): one bulk copy of CH packed weight tiles, one
  // 3-D TMA of CH activation tiles. A copy costs a fixed ~0.2 us of issue on its
  // thread, so copies must be >= ~16 KB for one issuing thread to keep up with HBM.
  static constexpr int CHMAX = X_BYTES <= 4096 ? 4 : X_BYTES <= 8192 ? 4 : X_BYTES <= 16384 ? 2 : 1;
  static constexpr int XSLOT = CHMAX * X_BYTES;   // one activation chunk
  static constexpr int XS = XSLOT <= 16384 ? 3 : 2;
  static constexpr int RAW_AVAIL = 208 * 1024 - WD * W_BYTES - XS * XSLOT;
  static constexpr int RD_ = RAW_AVAIL / RAW_BYTES > 24 ? 24 : RAW_AVAIL / RAW_BYTES;
  static constexpr int RD = RD_ - RD_ % 4;        // multiple of NG and of every chunk size
  static_assert(RD >= 8, "raw ring too shallow");
  static_assert(WD % NG == 0 && RPW % 16 == 0 && RD % CHMAX == 0, "ring / group shape");
  static constexpr int X_OFF = WD * W_BYTES;
  static constexpr int RAW_OFF = X_OFF + XS * XSLOT;
  static constexpr int BAR_OFF = ((RAW_OFF + RD * RAW_BYTES + 15) / 16) * 16;
  static constexpr int SMEM_BYTES = BAR_OFF + (2 * WD + 2 * XS + 2 * RD + 4) * 8 + 16 + 1024;
};

// One pair of 4-bit values (bits 0-3 and 16-19 of t) -> bf16x2 (q - 8) * s:
// (t & 0x000F000F) | bf16x2(128, 128) is exactly 128 + q per half, minus 136 is
// exact, and the scale multiply rounds once.
__device__ __forceinline__ uint32_t q4_pair(uint32_t t, uint32_t s2) {
  uint32_t v;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(v) : "r"(t));  // (t & m) | c
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  const uint32_t off = 0x43084308u;  // bf16x2(136, 136)
  b = __hsub2(b, *reinterpret_cast<const __nv_bfloat162*>(&off));
  b = __hmul2(b, *reinterpret_cast<const __nv_bfloat162*>(&s2));
  return *reinterpret_cast<uint32_t*>(&b);
}
// One Q4 word of the device format (k = 8w .. 8w+7: k = 8w+2i in bits [4i, 4i+4),
// k = 8w+2i+1 in bits [16+4i, 16+4i+4)) -> 8 consecutive bf16.
__device__ __forceinline__ uint4 q4_word(uint32_t w, uint32_t s2) {
  uint4 o;
  o.x = q4_pair(w, s2);
  o.y = q4_pair(w >> 4, s2);
  o.z = q4_pair(w >> 8, s2);
  o.w = q4_pair(w >> 12, s2);
  return o;
}
// Two offset-binary INT8 bytes (q + 128; bytes b0 and b0 + 1 of w) -> bf16x2 of q:
// the byte goes into the mantissa of 2^23 (exact), minus 2^23 + 128 (exact), then a
// packed conversion (exact for |q| <= 128).
__device__ __forceinline__ uint32_t i8_pair(uint32_t w, int b0) {
  const float lo = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650 + b0)) - 8388736.f;
  const float hi = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7651 + b0)) - 8388736.f;
  return pack_bf16x2(lo, hi);
}
__device__ __forceinline__ uint4 i8_chunk(uint32_t w0, uint32_t w1) {
  uint4 o;
  o.x = i8_pair(w0, 0);
  o.y = i8_pair(w0, 2);
  o.z = i8_pair(w1, 0);
  o.w = i8_pair(w1, 2);
  return o;
}


// Weight row-tiles of unit row-group tr (SWAP: g.rgroup consecutive 128-row
// tiles, the last group ragged; otherwise one).
__device__ __forceinline__ int unit_rows(const GemmArgs& g, int tr) {
  return g.swap ? min(g.rgroup, g.wt_tiles - tr * g.rgroup) : 1;
}

template <int BX, int QT, bool SWAP>
__global__ void __launch_bounds__(512, 1)
    gemm_wq_tc_kernel(const __grid_constant__ CUtensorMap tmX, const GemmArgs g) {
  using C = WqCfg<BX, QT, SWAP>;
  constexpr int BN_MMA = SWAP ? BX : 128;
  // SWAP: up to RMAX weight row-tiles share each activation tile (g.rgroup <= RMAX);
  // 2 x RMAX accumulators of BN_MMA columns (double-buffered across units).
  constexpr int RMAX = SWAP ? (256 / BN_MMA > 0 ? 256 / BN_MMA : 1) : 1;
  constexpr int TMEM_COLS = 2 * RMAX * BN_MMA < 32 ? 32 : 2 * RMAX * BN_MMA;
  constexpr int WD = C::WD, XS = C::XS, RD = C::RD;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wbuf = smem;
  uint8_t* xbuf = smem + C::X_OFF;
  uint8_t* rawbuf = smem + C::RAW_OFF;
  uint64_t* w_ready = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* w_empty = w_ready + WD;
  uint64_t* x_full = w_empty + WD;
  uint64_t* x_empty = x_full + XS;
  uint64_t* raw_full = x_empty + XS;   // one per chunk slot (index slot / CH)
  uint64_t* raw_empty = raw_full + RD; // one per tile slot
  uint64_t* tfull = raw_empty + RD;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = g.tiles_r * g.tiles_c * g.splits;
  const int CH = g.chunk;  // kb per chunk (divides every unit's kb count and RD)

  if (threadIdx.x == 0) {
    for (int s = 0; s < WD; ++s) {
      mbar_init(&w_ready[s], C::WPG);
      mbar_init(&w_empty[s], 1);
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < RD; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], C::WPG);
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

  // Tile order of a unit (every role walks it the same way): for each chunk c of CH
  // K blocks, for each of the unit's nR weight row-tiles j, the CH tiles (j, c*CH + kk).
  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int tr, tc, sp;
        unit_coords(g, u, tr, tc, sp);
        const int nR = unit_rows(g, tr);
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1 && ok; kb += CH) {
          for (int j = 0; j < nR && ok; ++j) {
            const int s0 = it % RD;  // chunk-aligned: it and RD are multiples of CH
            for (int q = 0; q < CH; ++q) {
              if (!mbar_wait(&raw_empty[s0 + q], (((it + q) / RD) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) {
                ok = false;
                break;
              }
            }
            if (!ok) break;
            const int wt = SWAP ? tr * g.rgroup + j : tc;  // weight tile (128 rows)
            uint64_t* fb = &raw_full[s0 / CH];
            mbar_arrive_expect_tx(fb, CH * C::RAW_BYTES);
            // CH consecutive K blocks of one pre-tiled weight row are contiguous: one copy
            bulk_load(rawbuf + s0 * C::RAW_BYTES, g.wtiles + ((size_t)wt * g.num_kb + kb) * C::RAW_BYTES,
                      CH * C::RAW_BYTES, fb);
            it += CH;
          }
        }
      }
      if (!ok) {  // drain the copies in flight before the CTA exits
        for (int j = max(0, it - RD); j < it; j += CH) mbar_wait(&raw_full[(j % RD) / CH], (j / RD) & 1, nullptr, 0);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ activation producer
    if (elect_one()) {
      int ix = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int tr, tc, sp;
        unit_coords(g, u, tr, tc, sp);
        const int xt = SWAP ? tc : tr;  // activation tile (BX rows)
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1; kb += CH, ++ix) {
          const int s = ix % XS;
          if (!mbar_wait(&x_empty[s], ((ix / XS) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          mbar_arrive_expect_tx(&x_full[s], CH * C::X_BYTES);
          // 3-D box {64 k, BX rows, CH k-blocks}: CH swizzled [BX][64] tiles back to back
          tma_load_3d(xbuf + s * C::XSLOT, &tmX, &x_full[s], 0, xt * BX, kb);
        }
      }
      if (!ok) {
        for (int j = max(0, ix - XS); j < ix; ++j) mbar_wait(&x_full[j % XS], (j / XS) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BN_MMA);
      int it = 0, ix = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++local) {
        int tr, tc, sp;
        unit_coords(g, u, tr, tc, sp);
        const int nR = unit_rows(g, tr);
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, g.status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
        tc_fence_after();
        for (int kb = kb0; kb < kb1 && ok; kb += CH, ++ix) {
          const int xs = ix % XS;
          if (!mbar_wait(&x_full[xs], (ix / XS) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          for (int j = 0; j < nR && ok; ++j) {
            const uint32_t d_tmem = tmem_base + (acc * RMAX + j) * BN_MMA;
            for (int kk = 0; kk < CH; ++kk, ++it) {
              const int ws = it % WD;
              if (!mbar_wait(&w_ready[ws], (it / WD) & 1, g.status, OM_ERR_WAIT_FULL)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t w_addr = smem_u32(wbuf + ws * C::W_BYTES);
              const uint32_t x_addr = smem_u32(xbuf + xs * C::XSLOT + kk * C::X_BYTES);
              const uint32_t a_addr = SWAP ? w_addr : x_addr;
              const uint32_t b_addr = SWAP ? x_addr : w_addr;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                tc_mma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32, 1024), smem_desc_sw128(b_addr + k * 32, 1024),
                           IDESC, (kb > kb0 || kk > 0 || k > 0) ? 1u : 0u);
              }
              tc_commit(&w_empty[ws]);
            }
          }
          if (ok) {
            tc_commit(&x_empty[xs]);
          }
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequant
    // Warp d is warp wi of group grp; per tile it expands rows [wi*RPW, wi*RPW + RPW)
    // in RPW/16 passes, lane -> (row pass*16 + lane / 2, half lane % 2 of the 64 k).
    constexpr int WPG = C::WPG, RPW = C::RPW, NG = C::NG, NP = RPW / 16;
    const int d = warp - 8;
    const int grp = d / WPG, wi = d % WPG;
    const int half = lane & 1;
    const uint32_t raw_s = smem_u32(rawbuf), w_s = smem_u32(wbuf);
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      int tr, tc, sp;
      unit_coords(g, u, tr, tc, sp);
      const int kb0 = sp * g.kb_per_split;
      const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
      const int nT = (kb1 - kb0) * unit_rows(g, tr);  // tiles of this unit, in producer order
      for (int t = 0; t < nT; ++t, ++it) {
        if (it % NG != grp) continue;
        const int r = it % RD, s = it % WD;
        if (!mbar_wait(&raw_full[r / CH], (it / RD) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
        const uint32_t raw = raw_s + r * C::RAW_BYTES;
        uint4 p0[NP] = {}, p1[NP] = {};
        uint32_t s2[NP] = {};
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          const int row = wi * RPW + j * 16 + (lane >> 1);
          if (QT == WQ_Q4) {
            // block `half` of the row: 16 bytes of nibbles (32 values) and its scale
            p0[j] = lds128(raw + row * 32 + half * 16);
            s2[j] = lds_u16(raw + C::RAW_Q + (half * 128 + row) * 2) * 0x10001u;
          } else {
            p0[j] = lds128(raw + row * 64 + half * 32);
            p1[j] = lds128(raw + row * 64 + half * 32 + 16);
          }
        }
        if (!mbar_wait(&w_empty[s], ((it / WD) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          const int row = wi * RPW + j * 16 + (lane >> 1);
          const uint32_t sw = row & 7;
          const uint32_t wrow = w_s + s * C::W_BYTES + row * 128;
          const uint32_t c0 = 4 * half;
          if (QT == WQ_Q4) {
            sts128(wrow + (((c0 + 0) ^ sw) << 4), q4_word(p0[j].x, s2[j]));
            sts128(wrow + (((c0 + 1) ^ sw) << 4), q4_word(p0[j].y, s2[j]));
            sts128(wrow + (((c0 + 2) ^ sw) << 4), q4_word(p0[j].z, s2[j]));
            sts128(wrow + (((c0 + 3) ^ sw) << 4), q4_word(p0[j].w, s2[j]));
          } else {
            sts128(wrow + (((c0 + 0) ^ sw) << 4), i8_chunk(p0[j].x, p0[j].y));
            sts128(wrow + (((c0 + 1) ^ sw) << 4), i8_chunk(p0[j].z, p0[j].w));
            sts128(wrow + (((c0 + 2) ^ sw) << 4), i8_chunk(p1[j].x, p1[j].y));
            sts128(wrow + (((c0 + 3) ^ sw) << 4), i8_chunk(p1[j].z, p1[j].w));
          }
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
      const int nR = unit_rows(g, tr);
      for (int j = 0; j < nR; ++j) {
        const int wt = SWAP ? tr * g.rgroup + j : tr;
        const int r = wt * 128 + q * 32 + lane;
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (acc * RMAX + j) * BN_MMA;
#pragma unroll 1
        for (int cc = 0; cc < BN_MMA / 32; ++cc) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + cc * 32, v);
          tc_wait_ld();
          epilogue_chunk(g, v, r, tc * BN_MMA + cc * 32, sp);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  if (g.po.pworld > 0) __threadfence_system();  // peer-output stores of this thread
  __syncthreads();
  peer_publish(g.po);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace om
