// Persistent warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   D[r, c] = sum_k A[r, k] * B[c, k]       (A: rows x K, B: cols x K, both K-major)
//
// Roles (256 threads, one CTA per SM):
//   warp 0      TMA producer: one elected lane streams 128x64 A tiles and
//               BNx64 B tiles (128-byte swizzle) into an S-stage smem ring.
//   warp 1      MMA issuer: one elected lane issues tcgen05.mma (M=128, N=BN,
//               K=16) into one of two TMEM accumulators, commits each stage back
//               to the producer and each finished tile to the epilogue.
//   warp 2      owns the TMEM allocation.
//   warps 4..7  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31), fuse residual add / split-K partial store, write.
// Two accumulators let the epilogue of tile i overlap the mainloop of tile i+1.
//
// "swap" mode computes Y^T: A is the weight, B the activations, and the
// epilogue writes Y[c][r]. It is the decode path (few tokens): the weight
// fills the 128-row MMA dimension and the token count becomes N (>= 32).
//
// Replaces the reference's scalar SIMT matmul and cuBLAS offload
// (openmini-server/src/kernel/cuda/kernels.cu:22-68,
//  openmini-server/src/hardware/gpu/cuda.rs:667-741,
//  openmini-server/src/model/inference/gemm_engine/cuda_backend.rs:72-87).
#pragma once
#include <cuda.h>
#include "gemm_common.cuh"

namespace om {

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
  // barriers + tmem slot live after the tiles
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256;
};

template <int BN>
__global__ void __launch_bounds__(256, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmArgs g) {
  using C = GemmCfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = g.tiles_r * g.tiles_c * g.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) tmem_alloc(tmem_slot, C::TMEM_COLS);
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
        const int kb0 = sp * g.kb_per_split;
        const int kb1 = min(g.num_kb, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, g.status, OM_ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* a_dst = tiles + s * C::STAGE_BYTES;
          uint8_t* b_dst = a_dst + C::A_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(a_dst, &tmA, &full[s], kb * C::BK, tr * C::BM);
          tma_load_2d(b_dst, &tmB, &full[s], kb * C::BK, tc * BN);
        }
      }
      if (!ok) {
        // drain: wait (bounded) for the loads that may still be in flight
        for (int j = max(0, it - C::STAGES); j < it; ++j)
          mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BN);
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
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, g.status, OM_ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(a_addr + k * 32, 1024);
            const uint64_t bd = smem_desc_sw128(b_addr + k * 32, 1024);
            tc_mma_f16(d_tmem, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter
    int local = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++local) {
      int tr, tc, sp;
      unit_coords(g, u, tr, tc, sp);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], aph, g.status, OM_ERR_WAIT_ACCUM)) break;
      tc_fence_after();
      const int r = tr * 128 + q * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + cc * 32, v);
        tc_wait_ld();
        epilogue_chunk(g, v, r, tc * BN + cc * 32, sp);
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
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace om
