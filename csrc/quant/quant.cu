// Weight-only quantisation formats used on the device.
//
// Q4 (GGUF Q4_0 semantics, block 32): per 32-element block one scale d and 16
// bytes of nibbles; byte i holds element i (low nibble) and element i + 16
// (high nibble); value = (q - 8) * d. On the device the scales are a separate
// bf16 array (the file's fp16 scale rounded once to bf16, so the dequantised
// weight is exactly representable in the bf16 MMA operand type). Quantiser:
// d = v_absmax_signed / -8, q = clamp(floor(v / d + 8.5), 0, 15) (the ggml
// reference quantiser). Restates the math of
// openmini-server/src/model/inference/quant.rs:121-215 (Q4_0), without its
// nibble-order quirk.
//
// INT8 (per output channel): q = round(v / s), s = absmax(row) / 127 (rounded
// to fp16), value = q * s; s kept in fp32 and applied in the GEMM epilogue.
// (openmini-server/src/kernel/cpu/quantized.rs:9-150 INT8 symmetric.)
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

__global__ void quantize_q4_kernel(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ q,
                                   __nv_bfloat16* __restrict__ scales, __half* __restrict__ scales_f16,
                                   size_t nblocks) {
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
    const __nv_bfloat16* src = w + b * 32;
    float v[32];
    float amax = 0.f, mx = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] = __bfloat162float(src[i]);
      if (fabsf(v[i]) > amax) {
        amax = fabsf(v[i]);
        mx = v[i];
      }
    }
    const __half dh = __float2half_rn(mx / -8.f);
    const __nv_bfloat16 db = __float2bfloat16_rn(__half2float(dh));
    const float d = __bfloat162float(db);
    const float id = d != 0.f ? 1.f / d : 0.f;
    uint8_t* dst = q + b * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      // separate multiply and add roundings (no FMA contraction) so the host quantiser matches bit for bit
      int lo = (int)floorf(__fadd_rn(__fmul_rn(v[i], id), 8.5f));
      int hi = (int)floorf(__fadd_rn(__fmul_rn(v[i + 16], id), 8.5f));
      lo = min(15, max(0, lo));
      hi = min(15, max(0, hi));
      dst[i] = (uint8_t)(lo | (hi << 4));
    }
    scales[b] = db;
    if (scales_f16) scales_f16[b] = dh;
  }
}

__global__ void dequant_q4_kernel(const uint8_t* __restrict__ q, const __nv_bfloat16* __restrict__ scales,
                                  __nv_bfloat16* __restrict__ out, size_t nblocks) {
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
    const uint4 pk = *reinterpret_cast<const uint4*>(q + b * 16);
    const float d = __bfloat162float(scales[b]);
    const uint8_t* by = reinterpret_cast<const uint8_t*>(&pk);
    float lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      lo[i] = (float)((int)(by[i] & 15) - 8) * d;
      hi[i] = (float)((int)(by[i] >> 4) - 8) * d;
    }
    uint4* o = reinterpret_cast<uint4*>(out + b * 32);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 u;
      u.x = pack_bf16x2(lo[8 * j + 0], lo[8 * j + 1]); u.y = pack_bf16x2(lo[8 * j + 2], lo[8 * j + 3]);
      u.z = pack_bf16x2(lo[8 * j + 4], lo[8 * j + 5]); u.w = pack_bf16x2(lo[8 * j + 6], lo[8 * j + 7]);
      o[j] = u;
      u.x = pack_bf16x2(hi[8 * j + 0], hi[8 * j + 1]); u.y = pack_bf16x2(hi[8 * j + 2], hi[8 * j + 3]);
      u.z = pack_bf16x2(hi[8 * j + 4], hi[8 * j + 5]); u.w = pack_bf16x2(hi[8 * j + 6], hi[8 * j + 7]);
      o[2 + j] = u;
    }
  }
}

// one block per row
__global__ void quantize_int8_kernel(const __nv_bfloat16* __restrict__ w, int8_t* __restrict__ q,
                                     float* __restrict__ scale, int K) {
  const int n = blockIdx.x;
  const __nv_bfloat16* row = w + (size_t)n * K;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(__bfloat162float(row[k])));
  __shared__ float sh[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) sh[0] = t;
  }
  __syncthreads();
  const float s = __half2float(__float2half_rn(sh[0] / 127.f));
  const float is = s > 0.f ? 1.f / s : 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = __bfloat162float(row[k]) * is;
    q[(size_t)n * K + k] = (int8_t)max(-127.f, min(127.f, rintf(v)));
  }
  if (threadIdx.x == 0) scale[n] = s;
}

__global__ void dequant_int8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                    __nv_bfloat16* __restrict__ out, int K, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn((float)q[i] * scale[i / K]);
}

}  // namespace om

static int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, (size_t)om::num_sms() * 32); }

void om_quantize_q4(torch::Tensor w, torch::Tensor q, torch::Tensor scales, c10::optional<torch::Tensor> scales_f16) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.size(-1) % 32 == 0, "quantize_q4: w");
  const size_t nb = w.numel() / 32;
  TORCH_CHECK((size_t)q.numel() == nb * 16 && (size_t)scales.numel() == nb, "quantize_q4: outputs");
  if (nb == 0) return;
  om::quantize_q4_kernel<<<grid_for(nb), 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), q.data_ptr<uint8_t>(),
      reinterpret_cast<__nv_bfloat16*>(scales.data_ptr()),
      scales_f16.has_value() ? reinterpret_cast<__half*>(scales_f16->data_ptr()) : nullptr, nb);
  OM_LAUNCH_CHECK();
}

void om_dequant_q4(torch::Tensor q, torch::Tensor scales, torch::Tensor out) {
  const size_t nb = scales.numel();
  TORCH_CHECK((size_t)q.numel() == nb * 16 && (size_t)out.numel() == nb * 32 && out.is_contiguous() &&
                  scales.is_contiguous(),
              "dequant_q4: shapes");
  if (nb == 0) return;
  om::dequant_q4_kernel<<<grid_for(nb), 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      q.data_ptr<uint8_t>(), reinterpret_cast<const __nv_bfloat16*>(scales.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nb);
  OM_LAUNCH_CHECK();
}

void om_quantize_int8(torch::Tensor w, torch::Tensor q, torch::Tensor scale) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 2, "quantize_int8: w");
  const int N = w.size(0), K = w.size(1);
  if (N == 0) return;
  om::quantize_int8_kernel<<<N, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), q.data_ptr<int8_t>(), scale.data_ptr<float>(), K);
  OM_LAUNCH_CHECK();
}

void om_dequant_int8(torch::Tensor q, torch::Tensor scale, torch::Tensor out) {
  const size_t n = q.numel();
  if (n == 0) return;
  om::dequant_int8_kernel<<<grid_for(n), 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      q.data_ptr<int8_t>(), scale.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), q.size(1),
      n);
  OM_LAUNCH_CHECK();
}
