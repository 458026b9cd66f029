// Shared pieces of the tcgen05 GEMM kernels: launch arguments, persistent
// tile order and the epilogue that turns one thread's 32 accumulator columns
// into output (bf16 store, residual add, per-weight-row scale, or fp32 split-K
// partial).
#pragma once
#include "../common/om_ptx.cuh"

namespace om {

enum GemmEpi : int { EPI_STORE = 0, EPI_RESID = 1, EPI_PARTIAL = 2 };

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
};

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
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, const uint32_t (&v)[32], int r, int c0, int sp) {
  if (r >= g.rows || c0 >= g.cols) return;
  const int ncol = min(32, g.cols - c0);
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
  if (g.wscale && g.epi != EPI_PARTIAL) {
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
  if (g.epi == EPI_PARTIAL) {
    float* P = reinterpret_cast<float*>(g.out);
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
  __nv_bfloat16* Y = reinterpret_cast<__nv_bfloat16*>(g.out);
  if (!g.swap) {
    __nv_bfloat16* dst = Y + (size_t)r * g.ldo + c0;
    const __nv_bfloat16* rs = g.resid ? g.resid + (size_t)r * g.ldo + c0 : nullptr;
    if (ncol == 32 && (g.ldo & 7) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = f[j + q];
        if (g.epi == EPI_RESID) {
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
          if (g.epi == EPI_RESID) t += __bfloat162float(rs[j]);
          dst[j] = __float2bfloat16_rn(t);
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < ncol) {
        const size_t o = (size_t)(c0 + j) * g.ldo + r;
        float t = f[j];
        if (g.epi == EPI_RESID) t += __bfloat162float(g.resid[o]);
        Y[o] = __float2bfloat16_rn(t);
      }
    }
  }
}

}  // namespace om
