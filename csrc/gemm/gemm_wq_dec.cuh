// Weight-only-quantised decode GEMM with the dequantised weight tile in tensor memory.
//
//   Y[t][n] = sum_k X[t][k] * dequant(W)[n][k],  t < M <= BX tokens (decode)
//
// The weight is the MMA's A operand (M = 128 weight rows), the tokens are N = BX.
// Dequant warps expand the packed tile straight into TENSOR memory with
// tcgen05.st and tcgen05.mma reads A from there (the "A in TMEM" form), so the
// bf16 weight never touches shared memory: shared memory only carries the packed
// weight (0.56 B per 4-bit weight) and the activation tile the MMA reads as B.
// Writing bf16 tiles to shared memory and reading them back through the MMA
// costs ~4.5 B of shared-memory traffic per weight, more than the SM's shared
// memory port delivers at HBM rate; that is what this layout removes.
//
// Stream-K schedule: the work items (row group g of R weight row-tiles, K chunk c
// of CH 64-wide K blocks) are numbered g-major and cut into gridDim.x equal
// contiguous ranges, so every CTA streams the same number of weight bytes
// whatever the tile count (no wave quantisation). A CTA accumulates each maximal
// run of items inside one group (a segment) in a TMEM accumulator; a segment that
// covers the whole K range goes straight to the output epilogue; a partial one
// (only the first and the last segment of a CTA can be partial) is stored as an
// fp32 slot (a CTA processes its two partial segments before its full ones, see
// SkOrder), and the CTA that completes a group's last segment (per-group counter)
// sums the group's slots in CTA order -- deterministic for a given shape -- and
// applies the final epilogue (per-row INT8 scale, residual, peer-output stores).
// No CTA ever waits for another one.
//
// Token halves: for 128 < M <= 256 the 128-token kernel runs every row group twice,
// once per half of the tokens (item group = row group * 2 + half), so a weight chunk
// is re-read from L2 right after its first use and the MMA stays 128 x 128.
//
// Fix-up of the CTA's last segment: when the CTA that completes a group does so in
// its final segment, nothing is left to overlap the fix-up with, so every warp of
// the CTA sums the slots (float4 over four weight rows, one token row of 512 bytes
// per warp and slot), instead of only the four epilogue warps.
//
// Handshakes are per raw chunk (CH K blocks = 16 MMAs of K = 16), not per K block:
// one issuing thread runs every MMA of the SM, and each wait / fence / commit it
// executes costs about as much as four MMAs, so a per-K-block handshake capped the
// whole kernel at ~3.4 TB/s (measured) while a bare bulk-copy ring of the same
// shape streams at HBM speed. The dequant warps likewise issue the CH tensor-memory
// stores of a chunk back to back and wait for them once.
//
// Roles (8 + 4 NG warps, one CTA per SM):
//   warp 0   bulk copies of the packed weight chunks (CH K blocks of one row-tile,
//            contiguous in the tiled device format) into the raw ring
//   warp 1   MMA issuer (one elected lane)
//   warp 2   TMEM allocation
//   warp 3   TMA of the activation chunks (3-D box: CH swizzled [BX][64] tiles)
//   4..7     epilogue (warp w reads TMEM lanes 32 (w % 4) ..)
//   8..      NG dequant groups of 4 warps; raw chunk t goes to group t % NG; warp
//            w of a group expands rows 32 (w % 4) + lane (one row per thread, the
//            TMEM lane quadrant a warp may access) into the group's own A slots.
//
// Q4 tile (128 rows x 64 k): per row 32 bytes, word w = k 8w..8w+7 with k = 8w+2i
// in bits [4i, 4i+4) and k = 8w+2i+1 in bits [16+4i, 16+4i+4); then the [2][128]
// bf16 block scales. Pair decode: (word >> 4i) & 0x000F000F | bf16x2(128, 128) is
// exactly (128 + q) per half; subtracting 136 is exact; one rounding in the scale
// multiply -- bit-identical to the shared-memory kernel.
// INT8 tile: 128 rows x 64 offset-binary bytes (q + 128); decode = byte into the
// mantissa of 2^23 (prmt), subtract 2^23 + 128 (exact), pack two to bf16x2
// (exact); the per-row scale is applied in the epilogue.
#pragma once
#include <cuda.h>
#include "gemm_common.cuh"
#include "gemm_wq.cuh"

namespace om {

template <int BX, int QT>
struct WqDecCfg {
  // weight row-tiles per group: every activation chunk brought in feeds R row-tiles
  static constexpr int R = BX == 32 ? 2 : 1;
  static constexpr int ACC_COLS = 2 * R * BX;               // double-buffered fp32 accumulators
  static constexpr int CH = QT == WQ_Q4 ? 4 : 2;            // K blocks per raw chunk
  static constexpr int NG = BX <= 64 ? 3 : 2;               // dequant groups
  static constexpr int NA = NG * CH;                        // A columns / 32 (group g owns CH kb at g * CH)
  static constexpr int TMEM_COLS = 512;
  static_assert(ACC_COLS + NA * 32 <= TMEM_COLS, "TMEM budget");
  static constexpr int THREADS = (8 + 4 * NG) * 32;
  static constexpr int RAW_Q = QT == WQ_Q4 ? 128 * 32 : 128 * 64;
  static constexpr int RAW = RAW_Q + (QT == WQ_Q4 ? 2 * 128 * 2 : 0);  // bytes per K block
  static constexpr int SLOT = CH * RAW;
  static constexpr int X_BYTES = BX * 64 * 2;
  static constexpr int XSLOT = CH * X_BYTES;
  static constexpr int XS = XSLOT <= 16384 ? 3 : 2;
  static constexpr int RS_ = (212 * 1024 - XS * XSLOT) / SLOT;
  static constexpr int RS = RS_ > 12 ? 12 : RS_;
  // A dequant group starts raw chunk u only after the MMA released the A slots of its
  // chunk u - NG, i.e. after the MMA consumed chunk u - 2 NG (so chunk u - 2 NG left
  // its raw slot). With RS >= 2 NG the chunk that last used u's raw slot (u - RS) is
  // then always consumed, and no group can wait on a raw-slot phase a full lap ahead
  // (which would alias the parity and pass the wait early).
  static_assert(RS >= 2 * NG, "raw ring shallower than two rounds of dequant groups");
  static constexpr int X_OFF = 0;
  static constexpr int RAW_OFF = XS * XSLOT;
  static constexpr int BAR_OFF = RAW_OFF + RS * SLOT;
  static constexpr int NBARS = 2 * XS + 2 * RS + 2 * NG + 4;
  static constexpr int STAGE_OFF = (BAR_OFF + NBARS * 8 + 16 + 127) / 128 * 128;
  static constexpr int STAGE_BYTES = 4 * 32 * 16 * 4;  // epilogue: per warp 32 rows x 16 tokens fp32
  static constexpr int SMEM_BYTES = STAGE_OFF + STAGE_BYTES + 1024;
};

// Output of one warp's 32 accumulator rows (weight rows rb .. rb + 31, one per lane,
// f = this lane's values for tokens c0 .. c0 + 31) to Y[token][row] (+ residual, with
// the INT8 per-row scale), in the transposed direction: through a 2 KB per-warp
// shared-memory stage, 16 tokens at a time, so each lane writes 8 consecutive rows of
// one token with one 16-byte store (a lane-per-row store is 2 bytes wide; 64 of them
// per thread measured ~11 us per segment under the full weight stream, the staged form
// is 8x fewer, 8x wider stores). vec = Y rows 16-byte aligned (host-checked); rows
// past the tensor and tokens past g.cols are skipped.
__device__ __forceinline__ void dec_store_rows(const GemmArgs& g, const float (&f)[32], int rb, int c0, float* stage,
                                               int epi, void* outp, const __nv_bfloat16* resid, bool vec) {
  const int lane = threadIdx.x & 31;
  const int r = rb + lane;
  const float sc = (g.wscale && r < g.rows) ? g.wscale[r] : 1.f;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 16; ++j) stage[j * 32 + lane] = f[hh * 16 + j] * sc;  // [token][row]
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int idx = it * 32 + lane;  // 16 tokens x 4 chunks of 8 rows
      const int jt = idx >> 2, ck = idx & 3;
      const int tok = c0 + hh * 16 + jt;
      const int row = rb + ck * 8;
      if (tok >= g.cols || row >= g.rows) continue;
      float v[8];
      const float4 a = *reinterpret_cast<const float4*>(stage + jt * 32 + ck * 8);
      const float4 b = *reinterpret_cast<const float4*>(stage + jt * 32 + ck * 8 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      __nv_bfloat16* dst = out_row(g, outp, tok) + row;
      const __nv_bfloat16* rs = epi == EPI_RESID ? resid + (size_t)tok * g.ldo + row : nullptr;
      if (vec && row + 8 <= g.rows) {
        if (rs) {
          float rv[8];
          unpack8(*reinterpret_cast<const uint4*>(rs), rv);
#pragma unroll
          for (int q = 0; q < 8; ++q) v[q] += rv[q];
        }
        *reinterpret_cast<uint4*>(dst) = pack8(v);
      } else {
        for (int q = 0; q < 8 && row + q < g.rows; ++q) {
          const float t = rs ? v[q] + __bfloat162float(rs[q]) : v[q];
          dst[q] = __float2bfloat16_rn(t);
        }
      }
    }
  }
}

// Final epilogue of four weight rows rr..rr+3 of token tok (values already summed, the
// INT8 per-row scales applied by the caller).
__device__ __forceinline__ void dec_store4(const GemmArgs& g, int tok, int rr, float4 v) {
  __nv_bfloat16* dst = out_row(g, g.out, tok) + rr;
  const __nv_bfloat16* rs = g.epi == EPI_RESID ? g.resid + (size_t)tok * g.ldo + rr : nullptr;
  if (g.vec_out && rr + 4 <= g.rows) {
    if (rs) {
      const uint2 r2 = *reinterpret_cast<const uint2*>(rs);
      v.x += bf16lo(r2.x); v.y += bf16hi(r2.x); v.z += bf16lo(r2.y); v.w += bf16hi(r2.y);
    }
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  } else {
    const float f[4] = {v.x, v.y, v.z, v.w};
    for (int q = 0; q < 4 && rr + q < g.rows; ++q)
      dst[q] = __float2bfloat16_rn(rs ? f[q] + __bfloat162float(rs[q]) : f[q]);
  }
}

// Sum of item group gg's fp32 slots (contributing CTAs c_lo..c_hi, in CTA order, so the
// result does not depend on which CTA finishes) and the final epilogue, by threads
// tid < nth (a multiple of 32): lane = four weight rows, warps stride over the tokens,
// U tokens per thread in flight per slot.
template <int BX, int R, int U>
__device__ void dec_fixup(const GemmArgs& g, long long gg, int grp, int half, int nR, int c_lo, int c_hi,
                          int tid, int nth) {
  const int NC = g.sk_nc;
  const long long T = g.sk_total, P = gridDim.x;
  const size_t slot_floats = (size_t)R * BX * 128;
  const int lane = tid & 31, w = tid >> 5, nw = nth >> 5;
  const int tok0 = half * BX;
  const int ntok = min(BX, g.cols - tok0);
  for (int j = 0; j < nR; ++j) {
    const int rr = (grp * R + j) * 128 + 4 * lane;
    float4 sc = make_float4(1.f, 1.f, 1.f, 1.f);
    if (g.wscale) {
      sc.x = rr < g.rows ? g.wscale[rr] : 1.f;
      sc.y = rr + 1 < g.rows ? g.wscale[rr + 1] : 1.f;
      sc.z = rr + 2 < g.rows ? g.wscale[rr + 2] : 1.f;
      sc.w = rr + 3 < g.rows ? g.wscale[rr + 3] : 1.f;
    }
    for (int t0 = w; t0 < ntok; t0 += nw * U) {
      float4 acc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c2 = c_lo; c2 <= c_hi; ++c2) {
        const long long b2 = (long long)c2 * T / P;
        const int sl = b2 / NC == gg ? 0 : 1;
        const float* src = g.part + ((size_t)c2 * 2 + sl) * slot_floats + (size_t)j * BX * 128 + 4 * lane;
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int t = t0 + u * nw;
          v[u] = t < ntok ? __ldcg(reinterpret_cast<const float4*>(src + (size_t)t * 128)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          acc[u].x += v[u].x; acc[u].y += v[u].y; acc[u].z += v[u].z; acc[u].w += v[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int t = t0 + u * nw;
        if (t >= ntok || rr >= g.rows) continue;
        const float4 o = make_float4(acc[u].x * sc.x, acc[u].y * sc.y, acc[u].z * sc.z, acc[u].w * sc.w);
        dec_store4(g, tok0 + t, rr, o);
      }
    }
  }
}

// A CTA's item range [ib, ie) in processing order: the partial head segment (items
// of the range's first group), then the partial tail segment (its last group), then
// the full groups in between. The two partial segments are the ones whose fp32 slots
// another CTA may have to sum, so producing them first lets that fix-up run early,
// overlapped with the streaming of the full groups, instead of at the end of the
// kernel (where it measured ~13 us of tail on the median CTA).
struct SkOrder {
  long long ib, ie, h_end, t_begin;
  __device__ __forceinline__ SkOrder(long long b, long long e, int NC) : ib(b), ie(e) {
    h_end = min(e, (b / NC + 1) * NC);
    t_begin = max(h_end, (e - 1) / NC * NC);
  }
  __device__ __forceinline__ long long n() const { return ie - ib; }
  __device__ __forceinline__ long long at(long long k) const {
    const long long nh = h_end - ib, nt = ie - t_begin;
    if (k < nh) return ib + k;
    if (k < nh + nt) return t_begin + (k - nh);
    return h_end + (k - nh - nt);
  }
};

template <int BX, int QT>
__global__ void __launch_bounds__(WqDecCfg<BX, QT>::THREADS, 1)
    gemm_wq_dec_kernel(const __grid_constant__ CUtensorMap tmX, const GemmArgs g) {
  using C = WqDecCfg<BX, QT>;
  constexpr int R = C::R, CH = C::CH, NG = C::NG, NA = C::NA, XS = C::XS, RS = C::RS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xbuf = smem + C::X_OFF;
  uint8_t* rawbuf = smem + C::RAW_OFF;
  uint64_t* x_full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* x_empty = x_full + XS;
  uint64_t* raw_full = x_empty + XS;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* a_full = raw_empty + RS;
  uint64_t* a_empty = a_full + NG;
  uint64_t* tfull = a_empty + NG;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  __shared__ int s_last;
  __shared__ long long s_fix[4];  // deferred fix-up of the final segment: gg, c_lo, c_hi, nR (gg < 0: none)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NC = g.sk_nc;
  const int NH = g.sk_nh;
  const long long T = g.sk_total;
  const long long P = gridDim.x;
  const long long ib = (long long)blockIdx.x * T / P;
  const long long ie = ((long long)blockIdx.x + 1) * T / P;
  const SkOrder ord(ib, ie, NC);
  const long long nk = ord.n();

  if (threadIdx.x == 0) {
    for (int s = 0; s < XS; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 4);
    }
    for (int s = 0; s < NG; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    s_fix[0] = -1;
    fence_barrier_init();
  }
  if (warp == 3 && lane == 0) tma_prefetch_desc(&tmX);
  if (warp == 2) tmem_alloc(tmem_slot, C::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ packed-weight producer
    if (elect_one()) {
      int t = 0;
      bool ok = true;
      for (long long k = 0; k < nk && ok; ++k) {
        const long long i = ord.at(k);
        const int grp = (int)(i / NC / NH), ch = (int)(i % NC);
        const int nR = min(R, g.wt_tiles - grp * R);
        for (int j = 0; j < nR; ++j, ++t) {
          const int s = t % RS;
          if (!mbar_poll(&raw_empty[s], ((t / RS) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          mbar_arrive_expect_tx(&raw_full[s], C::SLOT);
          bulk_load(rawbuf + s * C::SLOT,
                    g.wtiles + ((size_t)(grp * R + j) * g.num_kb + (size_t)ch * CH) * C::RAW, C::SLOT, &raw_full[s]);
        }
      }
      if (!ok)  // drain the copies in flight before the CTA exits
        for (int q = max(0, t - RS); q < t; ++q) mbar_wait(&raw_full[q % RS], (q / RS) & 1, nullptr, 0);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ activation producer
    if (elect_one()) {
      int ix = 0;
      bool ok = true;
      if (g.agwait_n > 0) {
        // the activations are the rows every rank pushed into this rank's gather region in
        // the previous sequence-parallel event: wait for all of them (bounded), then order
        // those generic-proxy peer writes before this warp's TMA (async-proxy) reads
        const int e = ld_volatile_s32(g.agwait + 32);
        const uint64_t t0 = globaltimer();
        for (int p = 0; p < g.agwait_n && ok; ++p) {
          uint32_t spins = 0;
          while (ld_acquire_sys_s32(g.agwait + 16 + p) < e) {
            if ((++spins & 63u) == 0 && globaltimer() - t0 > OM_WAIT_LIMIT_NS) {
              record_error(g.status, OM_ERR_WAIT_FULL);
              ok = false;
              break;
            }
          }
        }
        fence_proxy_async_global();
      }
      for (long long k = 0; k < nk && ok; ++k, ++ix) {
        const long long i = ord.at(k);
        const int ch = (int)(i % NC), half = (int)(i / NC % NH);
        const int s = ix % XS;
        if (!mbar_wait(&x_empty[s], ((ix / XS) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        mbar_arrive_expect_tx(&x_full[s], C::XSLOT);
        tma_load_3d(xbuf + s * C::XSLOT, &tmX, &x_full[s], 0, half * BX, ch * CH);
      }
      if (!ok)
        for (int q = max(0, ix - XS); q < ix; ++q) mbar_wait(&x_full[q % XS], (q / XS) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BX);
      int ix = 0, ta = 0, seg = 0;
      bool ok = true;
      for (long long k = 0; k < nk && ok; ++k, ++ix) {
        const long long i = ord.at(k);
        const int grp = (int)(i / NC / NH), ch = (int)(i % NC);
        const bool first = k == 0 || ch == 0 || ord.at(k - 1) != i - 1;
        const bool last = k == nk - 1 || ch == NC - 1 || ord.at(k + 1) != i + 1;
        const int nR = min(R, g.wt_tiles - grp * R);
        const int acc = seg & 1;
        if (first) {
          if (!mbar_poll(&tempty[acc], ((seg >> 1) & 1) ^ 1, g.status, OM_ERR_WAIT_ACCUM)) { ok = false; break; }
          tc_fence_after();
        }
        const int xs = ix % XS;
        if (!mbar_poll(&x_full[xs], (ix / XS) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
        tc_fence_after();
        const uint32_t x_addr = smem_u32(xbuf + xs * C::XSLOT);
        for (int j = 0; j < nR && ok; ++j, ++ta) {
          // raw chunk ta: expanded by group ta % NG into its CH A slots (one handshake per chunk)
          const int ga = ta % NG;
          if (!mbar_poll(&a_full[ga], (ta / NG) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (acc * R + j) * BX;
          const uint32_t a_tmem = tmem_base + C::ACC_COLS + ga * CH * 32;
#pragma unroll
          for (int kk = 0; kk < CH; ++kk)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_f16_ts(d_tmem, a_tmem + kk * 32 + k * 8, smem_desc_sw128(x_addr + kk * C::X_BYTES + k * 32, 1024),
                            IDESC, (first && kk == 0 && k == 0) ? 0u : 1u);
          tc_commit(&a_empty[ga]);
        }
        if (!ok) break;
        tc_commit(&x_empty[xs]);
        if (last) {
          tc_commit(&tfull[acc]);
          ++seg;
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequant into TMEM
    const int d = warp - 8;
    const int grp_id = d >> 2, quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t raw_s = smem_u32(rawbuf);
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    int t = 0;
    bool ok = true;
    for (long long k = 0; k < nk && ok; ++k) {
      const int grp = (int)(ord.at(k) / NC / NH);
      const int nR = min(R, g.wt_tiles - grp * R);
      for (int j = 0; j < nR; ++j, ++t) {
        if (t % NG != grp_id) continue;
        const int s = t % RS;
        if (!mbar_wait(&raw_full[s], (t / RS) & 1, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
        const uint32_t slot = raw_s + s * C::SLOT;
        // Stage the thread's whole row of the chunk in registers (the slot is released
        // after the tensor-memory stores below, behind a generic -> async proxy fence).
        constexpr int WPK = QT == WQ_Q4 ? 8 : 16;  // packed 32-bit words per row per K block
        uint32_t wr[CH][WPK];
        uint32_t sc[CH];  // Q4: the row's two bf16 block scales of each K block
#pragma unroll
        for (int kk = 0; kk < CH; ++kk) {
          const uint32_t base = slot + kk * C::RAW;
#pragma unroll
          for (int q = 0; q < WPK / 4; ++q) {
            const uint4 u = lds128(base + row * (WPK * 4) + q * 16);
            wr[kk][4 * q] = u.x; wr[kk][4 * q + 1] = u.y; wr[kk][4 * q + 2] = u.z; wr[kk][4 * q + 3] = u.w;
          }
          if (QT == WQ_Q4)
            sc[kk] = lds_u16(base + C::RAW_Q + row * 2) | (lds_u16(base + C::RAW_Q + 256 + row * 2) << 16);
        }

        // the group's A slots are free once the MMA finished this group's previous chunk
        if (!mbar_wait(&a_empty[grp_id], ((t / NG) & 1) ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_cols = tmem_base + lane_base + C::ACC_COLS + grp_id * CH * 32;
#pragma unroll
        for (int kk = 0; kk < CH; ++kk) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // 16 columns (32 k) per store
            uint32_t v[16];
            if (QT == WQ_Q4) {
              const uint32_t s2 = __byte_perm(sc[kk], 0, h ? 0x3232 : 0x1010);  // block h scale in both halves
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const uint4 o = q4_word(wr[kk][4 * h + w], s2);
                v[4 * w + 0] = o.x; v[4 * w + 1] = o.y; v[4 * w + 2] = o.z; v[4 * w + 3] = o.w;
              }
            } else {
#pragma unroll
              for (int w = 0; w < 8; ++w) {
                v[2 * w + 0] = i8_pair(wr[kk][8 * h + w], 0);
                v[2 * w + 1] = i8_pair(wr[kk][8 * h + w], 2);
              }
            }
            // the source registers are read when the store issues; one wait below covers all
            tmem_st_32x32b_x16(a_cols + kk * 32 + h * 16, v);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[grp_id]);
        // Release the raw slot only now, behind a proxy fence: the next bulk copy into it
        // is an async-proxy write, and without the fence it overwrote rows that the generic
        // loads above had not yet read (measured: INT8 outputs differed from run to run).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[s]);
        if (!ok) break;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int rl = quad * 32 + lane;  // accumulator lane = row within the weight tile
    float* stage = reinterpret_cast<float*>(smem + C::STAGE_OFF) + quad * 32 * 16;
    const bool vec_out = g.vec_out != 0;
    const size_t slot_floats = (size_t)R * BX * 128;
    int seg = 0, seg_ch0 = 0;
    for (long long k = 0; k < nk; ++k) {
      const long long i = ord.at(k);
      const long long gg = i / NC;
      const int grp = (int)(gg / NH), half = (int)(gg % NH), ch = (int)(i % NC);
      const int tok0 = half * BX;
      if (k == 0 || ch == 0 || ord.at(k - 1) != i - 1) seg_ch0 = ch;
      if (!(k == nk - 1 || ch == NC - 1 || ord.at(k + 1) != i + 1)) continue;
      const int nR = min(R, g.wt_tiles - grp * R);
      const int acc = seg & 1;
      if (!mbar_wait(&tfull[acc], (seg >> 1) & 1, g.status, OM_ERR_WAIT_ACCUM)) break;
      tc_fence_after();
      const bool full = seg_ch0 == 0 && ch == NC - 1;
      const int slot = gg == ib / NC ? 0 : 1;  // the range's first item group: slot 0
      float* mine = g.part + ((size_t)blockIdx.x * 2 + slot) * slot_floats;
      for (int j = 0; j < nR; ++j) {
        const int r = (grp * R + j) * 128 + rl;
        const uint32_t tb = tmem_base + ((uint32_t)(quad * 32) << 16) + (acc * R + j) * BX;
#pragma unroll 1
        for (int cc = 0; cc < BX / 32; ++cc) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tb + cc * 32, v);
          tc_wait_ld();
          if (tok0 + cc * 32 >= g.cols) continue;
          float f[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) f[q] = __uint_as_float(v[q]);
          if (full) {
            dec_store_rows(g, f, r - lane, tok0 + cc * 32, stage, g.epi, g.out, g.resid, vec_out);
          } else {
            float* dst = mine + (size_t)(j * BX + cc * 32) * 128 + rl;
#pragma unroll
            for (int q = 0; q < 32; ++q) dst[q * 128] = f[q];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (!full) {
        // counter protocol: the CTA that completes the group's last segment finishes it
        __threadfence();
        named_bar_sync(1, 128);
        const long long g0 = gg * NC, g1 = g0 + NC - 1;
        const int c_lo = (int)(((g0 + 1) * P + T - 1) / T - 1);
        const int c_hi = (int)(((g1 + 1) * P + T - 1) / T - 1);
        if (rl == 0) {
          const int prev = atomicAdd(&g.sem[gg], 1);
          s_last = prev == c_hi - c_lo;
          if (s_last) g.sem[gg] = 0;  // zero again for the next launch
        }
        named_bar_sync(1, 128);
        if (s_last) {
          __threadfence();
          if (k == nk - 1) {  // nothing left to overlap with: the whole CTA sums after the loop
            if (rl == 0) {
              s_fix[0] = gg;
              s_fix[1] = c_lo;
              s_fix[2] = c_hi;
              s_fix[3] = nR;
            }
          } else {
            dec_fixup<BX, R, 8>(g, gg, grp, half, nR, c_lo, c_hi, rl, 128);
          }
        }
      }
      ++seg;
    }
  }

  __syncthreads();
  if (s_fix[0] >= 0) {
    __threadfence();
    const long long gg = s_fix[0];
    dec_fixup<BX, R, 4>(g, gg, (int)(gg / NH), (int)(gg % NH), (int)s_fix[3], (int)s_fix[1], (int)s_fix[2],
                        threadIdx.x, C::THREADS);
  }
  if (g.po.pworld > 0) __threadfence_system();  // peer-output stores of this thread
  __syncthreads();
  peer_publish(g.po);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace om
