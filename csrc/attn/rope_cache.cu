// Rotary position embedding applied in place to the Q and K parts of the fused
// QKV projection output, fused with the write of K and V into the paged cache.
//
// Cache layout: [num_blocks, n_kv_heads, BLOCK=16, head_dim] bf16, so one
// (block, head) is a contiguous 16 x head_dim tile.
//
// Rotation modes:
//   0 interleaved pairs (2i, 2i+1), freq_i = theta^(-2i/head_dim): the GGUF
//     llama convention and the reference's apply_rotary_emb
//     (openmini-server/src/model/inference/model.rs:1108-1185,
//      openmini-server/src/kernel/cuda/kernels.cu:345-373)
//   1 half-split pairs (i, i + head_dim/2) ("neox" / HF checkpoints)
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

__global__ void rope_kv_kernel(__nv_bfloat16* __restrict__ qkv, int ld, const int* __restrict__ positions,
                               const int* __restrict__ slots, __nv_bfloat16* __restrict__ kc,
                               __nv_bfloat16* __restrict__ vc, const float* __restrict__ inv_freq, int Hq, int Hkv,
                               int D, int mode, int num_slots, int* status) {
  __shared__ float cs[2][128];
  const int t = blockIdx.x;
  const int pos = positions[t];
  const int half = D / 2;
  __nv_bfloat16* row = qkv + (size_t)t * ld;
  const int rot_heads = Hq + Hkv;
  // angles once per token, shared by all heads of this CTA
  for (int j = threadIdx.x; j < half; j += blockDim.x) sincosf((float)pos * inv_freq[j], &cs[0][j], &cs[1][j]);
  __syncthreads();
  // blockIdx.y splits the heads across CTAs
  const int hpb = (rot_heads + gridDim.y - 1) / gridDim.y;
  const int h0 = blockIdx.y * hpb, h1 = min(rot_heads, h0 + hpb);
  for (int i = threadIdx.x; i < (h1 - h0) * half; i += blockDim.x) {
    const int h = h0 + i / half, j = i % half;
    const float s = cs[0][j], c = cs[1][j];
    __nv_bfloat16* hp = row + h * D;
    const int i0 = mode == 0 ? 2 * j : j;
    const int i1 = mode == 0 ? 2 * j + 1 : j + half;
    const float x0 = __bfloat162float(hp[i0]), x1 = __bfloat162float(hp[i1]);
    hp[i0] = __float2bfloat16_rn(x0 * c - x1 * s);
    hp[i1] = __float2bfloat16_rn(x0 * s + x1 * c);
  }
  __syncthreads();
  const int slot = slots[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0 && blockIdx.y == 0) record_error(status, OM_ERR_BOUNDS);
    return;
  }
  const int blk = slot >> 4, off = slot & 15;
  const int nv = D / 8;
  for (int i = threadIdx.x; i < Hkv * nv; i += blockDim.x) {
    const int h = i / nv, c = i % nv;
    const size_t dst = (((size_t)blk * Hkv + h) * 16 + off) * D;
    // K heads are written by the CTA that rotated them, V heads by CTA y = 0
    if (Hq + h >= h0 && Hq + h < h1)
      reinterpret_cast<uint4*>(kc + dst)[c] = reinterpret_cast<const uint4*>(row + (Hq + h) * D)[c];
    if (blockIdx.y == 0)
      reinterpret_cast<uint4*>(vc + dst)[c] = reinterpret_cast<const uint4*>(row + (Hq + Hkv + h) * D)[c];
  }
}

// Write already-rotated K and V rows into the cache (used when K/V come from
// elsewhere, e.g. a prefix import or a ring-attention hop).
__global__ void kv_write_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, int ldk,
                                const int* __restrict__ slots, __nv_bfloat16* __restrict__ kc,
                                __nv_bfloat16* __restrict__ vc, int Hkv, int D) {
  const int t = blockIdx.x;
  const int slot = slots[t];
  if (slot < 0) return;
  const int blk = slot >> 4, off = slot & 15;
  const int nv = D / 8;
  for (int i = threadIdx.x; i < Hkv * nv; i += blockDim.x) {
    const int h = i / nv, c = i % nv;
    const size_t dst = (((size_t)blk * Hkv + h) * 16 + off) * D;
    reinterpret_cast<uint4*>(kc + dst)[c] = reinterpret_cast<const uint4*>(k + (size_t)t * ldk + h * D)[c];
    reinterpret_cast<uint4*>(vc + dst)[c] = reinterpret_cast<const uint4*>(v + (size_t)t * ldk + h * D)[c];
  }
}

}  // namespace om

void om_rope_kv(torch::Tensor qkv, torch::Tensor positions, torch::Tensor slots, torch::Tensor k_cache,
                torch::Tensor v_cache, torch::Tensor inv_freq, int64_t Hq, int64_t Hkv, int64_t D, int64_t mode,
                torch::Tensor status) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.stride(-1) == 1, "rope_kv: qkv");
  TORCH_CHECK(qkv.size(-1) >= (Hq + 2 * Hkv) * D && D % 8 == 0, "rope_kv: qkv width");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(1) == Hkv &&
                  k_cache.size(2) == 16 && k_cache.size(3) == D,
              "rope_kv: cache must be [blocks, Hkv, 16, D]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt, "rope_kv: int32 indices");
  TORCH_CHECK(inv_freq.scalar_type() == at::kFloat && inv_freq.numel() == D / 2, "rope_kv: inv_freq");
  const int T = positions.numel();
  if (T == 0) return;
  TORCH_CHECK(D / 2 <= 128, "rope_kv: head_dim <= 256");
  const int ysplit = std::max<int64_t>(1, std::min<int64_t>(8, (Hq + Hkv) / 8));
  om::rope_kv_kernel<<<dim3(T, ysplit), 128, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int>(),
      slots.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), inv_freq.data_ptr<float>(), Hq, Hkv, D, mode,
      k_cache.size(0) * 16, status.data_ptr<int>());
  OM_LAUNCH_CHECK();
}

void om_kv_write(torch::Tensor k, torch::Tensor v, torch::Tensor slots, torch::Tensor k_cache,
                 torch::Tensor v_cache) {
  const int T = slots.numel();
  if (T == 0) return;
  const int Hkv = k_cache.size(1), D = k_cache.size(3);
  TORCH_CHECK(k.stride(-1) == 1 && v.stride(0) == k.stride(0), "kv_write: layout");
  om::kv_write_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()),
      k.stride(0), slots.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), Hkv, D);
  OM_LAUNCH_CHECK();
}
