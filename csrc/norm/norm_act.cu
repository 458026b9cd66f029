// Row-wise normalisation, activation and small elementwise kernels (bf16 I/O,
// fp32 math), vectorised with 16-byte accesses.
//
// Reference ops restated here (math, not code):
//   RMSNorm     openmini-server/src/kernel/cuda/kernels.cu:291-322,
//               openmini-server/src/model/inference/model.rs:1067
//   LayerNorm   openmini-server/src/kernel/cuda/kernels.cu:149-206
//   GELU (tanh) openmini-server/src/kernel/cuda/kernels.cu:328-339
//   softmax     openmini-server/src/kernel/cuda/kernels.cu:77-140
//   SiLU gate   openmini-server/src/model/inference/gemm_engine.rs:98-130 (silu(gate)*up)
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = (l < NT / 32) ? sh[l] : 0.f;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}
template <int NT>
__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = (l < NT / 32) ? sh[l] : -INFINITY;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (l == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}


// out = rmsnorm(x [+ delta]) * w ; if delta != null, x is updated in place to x + delta.
// D % 8 == 0, D <= 8 * NT * VPT.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* delta,
                                                     const __nv_bfloat16* __restrict__ w,
                                                     __nv_bfloat16* __restrict__ out, int D, int ldx, int ldd,
                                                     int ldo, float eps) {
  __shared__ float sh[33];
  const int row = blockIdx.x;
  __nv_bfloat16* xr = x + (size_t)row * ldx;
  const int nv = D / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    if (c < nv) {
      uint4 u = reinterpret_cast<const uint4*>(xr)[c];
      unpack8(u, v[i]);
      if (delta) {
        float d[8];
        unpack8(reinterpret_cast<const uint4*>(delta + (size_t)row * ldd)[c], d);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[i][t] += d[t];
        uint4 nu = pack8(v[i]);
        reinterpret_cast<uint4*>(xr)[c] = nu;
        unpack8(nu, v[i]);  // normalise the rounded residual, as a separate add would
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) ss += v[i][t] * v[i][t];
    }
  }
  const float tot = block_sum<NT>(ss, sh);
  const float inv = rsqrtf(tot / D + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    if (c < nv) {
      float wf[8];
      unpack8(reinterpret_cast<const uint4*>(w)[c], wf);
      float o[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) o[t] = v[i][t] * inv * wf[t];
      reinterpret_cast<uint4*>(out + (size_t)row * ldo)[c] = pack8(o);
    }
  }
}

// LayerNorm with affine (bias optional). One block per row; fp32 two-pass.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) layernorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       const __nv_bfloat16* __restrict__ b,
                                                       __nv_bfloat16* __restrict__ out, int D, float eps) {
  __shared__ float sh[33];
  const int row = blockIdx.x;
  const int nv = D / 8;
  float v[VPT][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    if (c < nv) {
      unpack8(reinterpret_cast<const uint4*>(x + (size_t)row * D)[c], v[i]);
#pragma unroll
      for (int t = 0; t < 8; ++t) s += v[i][t];
    }
  }
  const float mean = block_sum<NT>(s, sh) / D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    if (c < nv) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        float d = v[i][t] - mean;
        q += d * d;
      }
    }
  }
  const float inv = rsqrtf(block_sum<NT>(q, sh) / D + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    if (c < nv) {
      float wf[8], bf[8] = {0, 0, 0, 0, 0, 0, 0, 0}, o[8];
      unpack8(reinterpret_cast<const uint4*>(w)[c], wf);
      if (b) unpack8(reinterpret_cast<const uint4*>(b)[c], bf);
#pragma unroll
      for (int t = 0; t < 8; ++t) o[t] = (v[i][t] - mean) * inv * wf[t] + bf[t];
      reinterpret_cast<uint4*>(out + (size_t)row * D)[c] = pack8(o);
    }
  }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

// out[t, f] = silu(gu[t, f]) * gu[t, F + f]   (gate half first, then up half)
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int T,
                                int F) {
  const int nv = F / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)T * nv;
       i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / nv), c = (int)(i % nv);
    const uint4* row = reinterpret_cast<const uint4*>(gu + (size_t)t * 2 * F);
    float g[8], u[8], o[8];
    unpack8(row[c], g);
    unpack8(row[nv + c], u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = silu_f(g[k]) * u[k];
    reinterpret_cast<uint4*>(out + (size_t)t * F)[c] = pack8(o);
  }
}

// tanh-approximation GELU, elementwise
__global__ void gelu_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, size_t n8) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    float f[8], o[8];
    unpack8(reinterpret_cast<const uint4*>(x)[i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float a = f[k];
      o[k] = 0.5f * a * (1.f + tanhf(0.7978845608028654f * (a + 0.044715f * a * a * a)));
    }
    reinterpret_cast<uint4*>(y)[i] = pack8(o);
  }
}

// row softmax, fp32 output, one block per row
template <int NT>
__global__ void softmax_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y, int D, float scale) {
  __shared__ float sh[33];
  const __nv_bfloat16* xr = x + (size_t)blockIdx.x * D;
  float* yr = y + (size_t)blockIdx.x * D;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < D; i += NT) m = fmaxf(m, __bfloat162float(xr[i]) * scale);
  m = block_max<NT>(m, sh);
  float s = 0.f;
  for (int i = threadIdx.x; i < D; i += NT) s += __expf(__bfloat162float(xr[i]) * scale - m);
  s = block_sum<NT>(s, sh);
  const float inv = 1.f / s;
  for (int i = threadIdx.x; i < D; i += NT) yr[i] = __expf(__bfloat162float(xr[i]) * scale - m) * inv;
}

// out[t] = table[ids[t]] (rows of D bf16); ids outside [0, V) yield zeros and flag the status word.
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int D, int V, int* status) {
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0) record_error(status, OM_ERR_BOUNDS);
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)(ok ? id : 0) * D);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * D);
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

}  // namespace om

using namespace om;

static void check_bf16(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, n, ": CUDA bf16 tensor required");
}

void om_rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> delta, torch::Tensor w, torch::Tensor out,
                double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  const int D = x.size(-1);
  const int T = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 8 * 256 * 8, "rmsnorm: D must be a multiple of 8 and <= 16384");
  TORCH_CHECK(x.stride(-1) == 1 && out.stride(-1) == 1, "rmsnorm: inner dim contiguous");
  if (T == 0) return;
  const __nv_bfloat16* dp = nullptr;
  int ldd = D;
  if (delta.has_value()) {
    check_bf16(*delta, "delta");
    TORCH_CHECK(delta->numel() == x.numel() && delta->stride(-1) == 1, "rmsnorm: delta layout");
    dp = reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr());
    ldd = delta->dim() >= 2 ? delta->stride(-2) : D;
  }
  const int ldx = x.dim() >= 2 ? x.stride(-2) : D;
  const int ldo = out.dim() >= 2 ? out.stride(-2) : D;
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto xp = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (D <= 8 * 128 * 4)
    rmsnorm_kernel<128, 4><<<T, 128, 0, st>>>(xp, dp, wp, op, D, ldx, ldd, ldo, (float)eps);
  else
    rmsnorm_kernel<256, 8><<<T, 256, 0, st>>>(xp, dp, wp, op, D, ldx, ldd, ldo, (float)eps);
  OM_LAUNCH_CHECK();
}

void om_layernorm(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, torch::Tensor out,
                  double eps) {
  check_bf16(x, "x");
  const int D = x.size(-1);
  const int T = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 16384 && x.is_contiguous() && out.is_contiguous(), "layernorm: layout");
  if (T == 0) return;
  auto st = at::cuda::getCurrentCUDAStream().stream();
  layernorm_kernel<256, 8><<<T, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      b.has_value() ? reinterpret_cast<const __nv_bfloat16*>(b->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D, (float)eps);
  OM_LAUNCH_CHECK();
}

void om_silu_mul(torch::Tensor gu, torch::Tensor out) {
  check_bf16(gu, "gu");
  check_bf16(out, "out");
  const int F = out.size(-1);
  const int T = out.numel() / F;
  TORCH_CHECK(gu.size(-1) == 2 * F && F % 8 == 0 && gu.is_contiguous() && out.is_contiguous(), "silu_mul: layout");
  const size_t work = (size_t)T * (F / 8);
  if (work == 0) return;
  const int blocks = (int)std::min<size_t>((work + 255) / 256, (size_t)num_sms() * 16);
  silu_mul_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, F);
  OM_LAUNCH_CHECK();
}

void om_gelu(torch::Tensor x, torch::Tensor y) {
  check_bf16(x, "x");
  TORCH_CHECK(x.numel() % 8 == 0 && x.is_contiguous() && y.is_contiguous(), "gelu: layout");
  const size_t n8 = x.numel() / 8;
  if (n8 == 0) return;
  const int blocks = (int)std::min<size_t>((n8 + 255) / 256, (size_t)num_sms() * 16);
  gelu_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n8);
  OM_LAUNCH_CHECK();
}

void om_softmax(torch::Tensor x, torch::Tensor y, double scale) {
  check_bf16(x, "x");
  TORCH_CHECK(y.scalar_type() == at::kFloat && x.is_contiguous() && y.is_contiguous(), "softmax: layout");
  const int D = x.size(-1);
  const int T = x.numel() / D;
  if (T == 0) return;
  softmax_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), y.data_ptr<float>(), D, (float)scale);
  OM_LAUNCH_CHECK();
}

void om_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, torch::Tensor status) {
  check_bf16(table, "table");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_cuda(), "embedding: int32 ids");
  const int T = ids.numel(), D = table.size(1);
  TORCH_CHECK(D % 8 == 0 && table.is_contiguous() && out.is_contiguous(), "embedding: layout");
  if (T == 0) return;
  embedding_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D, table.size(0), status.data_ptr<int>());
  OM_LAUNCH_CHECK();
}
