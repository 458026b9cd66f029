// Shared pieces of the tcgen05 GEMM kernels: launch arguments, persistent
// tile order and the epilogue that turns one thread's 32 accumulator columns
// into output (bf16 store, residual add, per-weight-row scale, or fp32 split-K
// partial).
#pragma once
#include "../common/om_ptx.cuh"

namespace om {

enum GemmEpi : int { EPI_STORE = 0, EPI_RESID = 1, EPI_PARTIAL = 2 };

// Peer output (tensor-parallel GEMM -> reduce-scatter in one kernel). With
// pworld > 0, row m of Y goes to the owner rank o = m / rows_own, into slot
// `prank` of its partials region: peer[o] + peer_off + ((prank * rows_own +
// m % rows_own) * ldo + n) * 2 bytes, stored over NVLink (plain st.global to a
// CUDA-IPC mapping of the peer's buffer) as the tile leaves TMEM. The last CTA
// to finish then publishes the epoch (peer_publish).
struct PeerOut {
  uint8_t* peer[8];
  long long peer_off;
  int rows_own, prank, pworld;
};

__device__ __forceinline__ __nv_bfloat16* peer_row(const PeerOut& p, int ldo, int m) {
  const int o = m / p.rows_own;
  const int lr = m - o * p.rows_own;
  return reinterpret_cast<__nv_bfloat16*>(p.peer[o] + p.peer_off) + (size_t)(p.prank * p.rows_own + lr) * ldo;
}

// End-of-kernel publication of a peer-output kernel. Control words of the
// symmetric buffer (byte offsets): ready[8] at 0, epoch at 128, GEMM ticket at
// 136. Every thread has fenced its peer stores at system scope before the CTA
// barrier that precedes this call; thread 0 of the last CTA bumps the epoch
// and writes ready[prank] = epoch on every rank with release semantics.
__device__ __forceinline__ void peer_publish(const PeerOut& po) {
  if (po.pworld <= 0 || threadIdx.x != 0) return;
  uint8_t* own = po.peer[po.prank];
  unsigned* ticket = reinterpret_cast<unsigned*>(own + 136);
  const unsigned t = atomicAdd(ticket, 1u);
  if (t != gridDim.x - 1) return;
  *ticket = 0u;
  int* ep = reinterpret_cast<int*>(own + 128);
  const int e = *ep + 1;
  *ep = e;
  __threadfence_system();
  for (int p = 0; p < po.pworld; ++p) {
    int* f = reinterpret_cast<int*>(po.peer[p]) + po.prank;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
  }
}

struct GemmArgs {
  int rows;          // MMA M extent (rows of A)
  int cols;          // MMA N extent (rows of B)
  int num_kb;        // number of 64-wide K blocks
  int splits;        // split-K factor (>=1)
  int kb_per_split;  // K blocks per split
  int tiles_r, tiles_c;
  int swap;          // 1: output is Y[c][r] (A = weight, B = activations)
  int epi;           // GemmEpi
  void* out;         // bf16 Y (EPI_STORE/EPI_RESID) or fp32 partials [splits][Ym][Yn]
  const __nv_bfloat16* resid;  // EPI_RESID: Y += resid (may alias out)
  const float* wscale;         // optional per-weight-row scale (INT8 weights)
  const uint8_t* wtiles;       // quantised weights, pre-tiled (weight-only GEMM)
  int ldo;           // leading dimension of Y / resid (elements)
  int* status;
  int rgroup;        // weight-only SWAP: weight row-tiles per unit (tiles_r counts groups)
  int wt_tiles;      // weight-only: number of 128-row weight tiles
  int chunk;         // weight-only: K blocks per copy chunk (divides num_kb and kb_per_split)
  // Stream-K decode kernel: per-row-group counters of finished segments (zeroed
  // before the first launch; the finishing CTA zeroes its group's counter again).
  int* sem;
  PeerOut po;        // peer output (po.pworld > 0), see PeerOut
  // Stream-K decode kernel (gemm_wq_dec.cuh): the sk_total work items (row group,
  // K chunk) are cut into gridDim.x equal contiguous ranges; sk_nc chunks per group;
  // part = fp32 partial slots [gridDim.x][2][rgroup * 128 * cols_pad].
  long long sk_total;
  int sk_nc;
  const int* agwait;  // sequence-parallel gather to wait for before the first activation load:
  int agwait_n;       // this rank's symmetric control words (agdone[p] at byte 64, epoch at 128), ranks
  int sk_nh;         // token halves of BX tokens (2 when 128 < M <= 256): item group = row group * sk_nh + half
  float* part;
  int vec_out;       // output rows (and residual rows) 16-byte aligned: vector epilogue stores
};

// Row pointer of output row m (local Y, or the owner's slot in peer mode).
__device__ __forceinline__ __nv_bfloat16* out_row(const GemmArgs& g, void* out, int m) {
  if (g.po.pworld > 0) return peer_row(g.po, g.ldo, m);
  return reinterpret_cast<__nv_bfloat16*>(out) + (size_t)m * g.ldo;
}

__device__ __forceinline__ void unit_coords(const GemmArgs& g, int u, int& tr, int& tc, int& sp) {
  sp = u % g.splits;
  const int t = u / g.splits;
  // group-of-8 rasterisation along rows for L2 reuse of B tiles
  constexpr int GROUP = 8;
  const int per_group = GROUP * g.tiles_c;
  const int grp = t / per_group;
  const int first_r = grp * GROUP;
  const int gsize = min(GROUP, g.tiles_r - first_r);
  const int in = t % per_group;
  tr = first_r + (in % gsize);
  tc = in / gsize;
}

// Thread owns accumulator row r (global MMA row), columns c0 .. c0+31.
// One thread's 32 accumulator columns f of row r -> output, with the epilogue kind,
// output and residual given explicitly (the split-K finisher passes the final ones).
__device__ __forceinline__ void epilogue_f(const GemmArgs& g, float (&f)[32], int r, int c0, int sp, int epi,
                                           void* outp, const __nv_bfloat16* resid) {
  if (r >= g.rows || c0 >= g.cols) return;
  const int ncol = min(32, g.cols - c0);
  if (g.wscale && epi != EPI_PARTIAL) {
    if (g.swap) {
      const float s = g.wscale[r];
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] *= s;
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncol) f[j] *= g.wscale[c0 + j];
    }
  }
  if (epi == EPI_PARTIAL) {
    float* P = reinterpret_cast<float*>(outp);
    if (!g.swap) {
      float* dst = P + ((size_t)sp * g.rows + r) * g.cols + c0;
      if (ncol == 32 && (g.cols & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncol) dst[j] = f[j];
      }
    } else {
      float* dst = P + (size_t)sp * g.rows * g.cols;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncol) dst[(size_t)(c0 + j) * g.rows + r] = f[j];
    }
    return;
  }
  if (!g.swap) {
    __nv_bfloat16* dst = out_row(g, outp, r) + c0;
    const __nv_bfloat16* rs = resid ? resid + (size_t)r * g.ldo + c0 : nullptr;
    if (ncol == 32 && (g.ldo & 7) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = f[j + q];
        if (epi == EPI_RESID) {
          const uint4 rv = *reinterpret_cast<const uint4*>(rs + j);
          t[0] += bf16lo(rv.x); t[1] += bf16hi(rv.x); t[2] += bf16lo(rv.y); t[3] += bf16hi(rv.y);
          t[4] += bf16lo(rv.z); t[5] += bf16hi(rv.z); t[6] += bf16lo(rv.w); t[7] += bf16hi(rv.w);
        }
        uint4 o;
        o.x = pack_bf16x2(t[0], t[1]); o.y = pack_bf16x2(t[2], t[3]);
        o.z = pack_bf16x2(t[4], t[5]); o.w = pack_bf16x2(t[6], t[7]);
        *reinterpret_cast<uint4*>(dst + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < ncol) {
          float t = f[j];
          if (epi == EPI_RESID) t += __bfloat162float(rs[j]);
          dst[j] = __float2bfloat16_rn(t);
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < ncol) {
        float t = f[j];
        if (epi == EPI_RESID) t += __bfloat162float(resid[(size_t)(c0 + j) * g.ldo + r]);
        out_row(g, outp, c0 + j)[r] = __float2bfloat16_rn(t);
      }
    }
  }
}

__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, const uint32_t (&v)[32], int r, int c0, int sp) {
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
  epilogue_f(g, f, r, c0, sp, g.epi, g.out, g.resid);
}

}  // namespace om
