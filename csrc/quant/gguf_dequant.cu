// GGUF block formats -> bf16 on the device, for loading checkpoints without a host
// dequantisation pass: the packed tensor is copied to the GPU as is (0.5 - 1.1 bytes
// per weight) and expanded here, one thread per output element reading its block's
// scale bytes (cached) and its own quant bits.
//
// Layouts (public GGUF specification; little endian, fp16 scales):
//   Q4_0  32 el / 18 B: d | 16 B nibbles (element j < 16 low nibble of byte j, j >= 16 high
//                       nibble of byte j - 16); x = (q - 8) d
//   Q8_0  32 el / 34 B: d | 32 int8;                         x = q d
//   Q4_K 256 el / 144 B: d | dmin | 12 B 6-bit scales / mins | 128 B nibbles;
//                       sub-block j = e / 32 reads nibble (j % 2) of byte (j / 2) 32 + e % 32
//   Q5_K 256 el / 176 B: as Q4_K plus 32 B of 5th bits (bit j of qh[e % 32]) before the nibbles
//   Q6_K 256 el / 210 B: 128 B low nibbles | 64 B high 2-bit pairs | 16 int8 scales | d;
//                       x = d scale[e / 16] (q - 32)
//
// Reference counterpart: the SIMD dequantisers of openmini-server/src/model/inference/
// quant_simd.rs and quant.rs (host-side there).
#include "../common/om_host.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace om {

enum GgufType : int { GG_Q4_0 = 2, GG_Q8_0 = 8, GG_Q4_K = 12, GG_Q5_K = 13, GG_Q6_K = 14 };

__device__ __forceinline__ float ld_f16(const uint8_t* p) {
  const unsigned short u = (unsigned short)p[0] | ((unsigned short)p[1] << 8);
  return __half2float(__ushort_as_half(u));
}

__device__ __forceinline__ void k_scale_min(const uint8_t* sc, int j, int& s, int& m) {
  if (j < 4) {
    s = sc[j] & 63;
    m = sc[j + 4] & 63;
  } else {
    s = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4);
    m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
}

template <int TYPE>
__global__ void gguf_dequant_kernel(const uint8_t* __restrict__ raw, __nv_bfloat16* __restrict__ out, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float x;
  if (TYPE == GG_Q4_0) {
    const uint8_t* b = raw + (i >> 5) * 18;
    const int e = i & 31;
    const int q = e < 16 ? (b[2 + e] & 15) : (b[2 + e - 16] >> 4);
    x = (float)(q - 8) * ld_f16(b);
  } else if (TYPE == GG_Q8_0) {
    const uint8_t* b = raw + (i >> 5) * 34;
    x = (float)(int8_t)b[2 + (i & 31)] * ld_f16(b);
  } else if (TYPE == GG_Q4_K || TYPE == GG_Q5_K) {
    const int bytes = TYPE == GG_Q4_K ? 144 : 176;
    const uint8_t* b = raw + (i >> 8) * bytes;
    const int e = i & 255, j = e >> 5, l = e & 31;
    int s, m;
    k_scale_min(b + 4, j, s, m);
    const uint8_t* qs = b + (TYPE == GG_Q4_K ? 16 : 48);
    int q = (qs[(j >> 1) * 32 + l] >> (4 * (j & 1))) & 15;
    if (TYPE == GG_Q5_K) q += 16 * ((b[16 + l] >> j) & 1);
    x = ld_f16(b) * (float)s * (float)q - ld_f16(b + 2) * (float)m;
  } else {  // Q6_K
    const uint8_t* b = raw + (i >> 8) * 210;
    const int e = i & 255, h = e >> 7, r = e & 127, p = r >> 5, l = r & 31;
    const uint8_t* L = b + 64 * h;
    const uint8_t* H = b + 128 + 32 * h;
    const int lo = (p & 1) ? L[l + 32] : L[l];
    const int q = (((p & 2) ? (lo >> 4) : (lo & 15)) | (((H[l] >> (2 * p)) & 3) << 4)) - 32;
    x = ld_f16(b + 208) * (float)(int8_t)b[192 + (e >> 4)] * (float)q;
  }
  out[i] = __float2bfloat16_rn(x);
}

}  // namespace om

// raw: uint8 bytes of n elements of GGUF type `type` (on the device); out: bf16 [n].
void om_gguf_dequant(torch::Tensor raw, int64_t type, torch::Tensor out) {
  TORCH_CHECK(raw.is_cuda() && raw.scalar_type() == at::kByte && raw.is_contiguous(), "gguf_dequant: raw bytes");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "gguf_dequant: out bf16");
  const long long n = out.numel();
  int per, bytes;
  switch (type) {
    case om::GG_Q4_0: per = 32; bytes = 18; break;
    case om::GG_Q8_0: per = 32; bytes = 34; break;
    case om::GG_Q4_K: per = 256; bytes = 144; break;
    case om::GG_Q5_K: per = 256; bytes = 176; break;
    case om::GG_Q6_K: per = 256; bytes = 210; break;
    default: TORCH_CHECK(false, "gguf_dequant: type ", type, " is not decoded on the device");
  }
  TORCH_CHECK(n % per == 0 && raw.numel() >= n / per * bytes, "gguf_dequant: ", n, " elements need ",
              n / per * bytes, " bytes");
  if (n == 0) return;
  const int threads = 256;
  const unsigned grid = (unsigned)((n + threads - 1) / threads);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  const uint8_t* r = raw.data_ptr<uint8_t>();
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  switch (type) {
    case om::GG_Q4_0: om::gguf_dequant_kernel<om::GG_Q4_0><<<grid, threads, 0, st>>>(r, o, n); break;
    case om::GG_Q8_0: om::gguf_dequant_kernel<om::GG_Q8_0><<<grid, threads, 0, st>>>(r, o, n); break;
    case om::GG_Q4_K: om::gguf_dequant_kernel<om::GG_Q4_K><<<grid, threads, 0, st>>>(r, o, n); break;
    case om::GG_Q5_K: om::gguf_dequant_kernel<om::GG_Q5_K><<<grid, threads, 0, st>>>(r, o, n); break;
    default: om::gguf_dequant_kernel<om::GG_Q6_K><<<grid, threads, 0, st>>>(r, o, n); break;
  }
  OM_LAUNCH_CHECK();
}
