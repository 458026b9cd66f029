// Token sampler: temperature -> top-k -> top-p -> draw, one CTA per row.
//
// The reference sampler (openmini-server/src/model/inference/sampler.rs:220-450,
// openmini-server/src/model/inference/model.rs:3970) sorts the vocabulary. Here
// the top-k and top-p cut-offs are found without sorting by an MSB-first radix
// select over order-preserving 32-bit keys of the scaled logits (4 passes of
// 8-bit histograms in shared memory): counts for top-k, probability mass for
// top-p (the smallest prefix, in descending order, whose mass reaches p; ties
// at the cut-off are kept). The draw is a Gumbel-max race among the kept tokens
// with Philox-4x32-10 counter-based uniforms (Salmon et al., SC'11), so a
// (seed, offset) pair reproduces the draw exactly.
//
// Outputs: the token, its log-probability under the temperature-scaled full
// distribution, and optionally the kept set as a bitmask (bit i of word i/32)
// for sampling-mask replay in RL training.
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

template <typename T>
__device__ __forceinline__ float ld_logit(const T* p, int i);
template <>
__device__ __forceinline__ float ld_logit<float>(const float* p, int i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_logit<__nv_bfloat16>(const __nv_bfloat16* p, int i) {
  return __bfloat162float(p[i]);
}

struct SampleArgs {
  const void* logits;
  int ld, V;
  const float* temperature;
  const float* top_p;
  const int* top_k;
  const int64_t* rng;  // [B, 2] = (seed, offset)
  int* out_tok;
  float* out_logprob;
  uint32_t* keep_mask;  // [B, ceil(V/32)] or null
};

constexpr int SNT = 1024;

template <int NT>
__device__ __forceinline__ float bsum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < NT / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}

// Radix select over keys of x = logit/T - max. mode 0: largest cutoff with
// count(key >= cutoff) >= target. mode 1: largest cutoff with
// mass(key >= cutoff) >= target, restricted to keys >= floor_key.
template <typename T>
__device__ uint32_t radix_cutoff(const T* row, int V, float inv_t, float mx, int mode, float target,
                                 uint32_t floor_key, float* hist /*256*/, float* sh) {
  uint32_t prefix = 0, pmask = 0;
  float above = 0.f;  // count / mass of elements strictly above the chosen prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += SNT) hist[i] = 0.f;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += SNT) {
      const float x = ld_logit<T>(row, i) * inv_t - mx;
      const uint32_t k = f2key(x);
      if (k < floor_key) continue;
      if ((k & pmask) != prefix) continue;
      const float w = mode == 0 ? 1.f : __expf(x);
      atomicAdd(&hist[(k >> shift) & 255u], w);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float acc = above;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= target) break;
        acc += hist[d];
      }
      sh[40] = acc;
      sh[41] = __int_as_float(d);
    }
    __syncthreads();
    above = sh[40];
    const uint32_t d = (uint32_t)__float_as_int(sh[41]);
    prefix |= d << shift;
    pmask |= 255u << shift;
    __syncthreads();
  }
  return prefix;
}

template <typename T>
__global__ void __launch_bounds__(SNT) sample_kernel(const SampleArgs a) {
  __shared__ float sh[48];
  __shared__ float hist[256];
  __shared__ unsigned long long best;
  const int b = blockIdx.x;
  const T* row = reinterpret_cast<const T*>(a.logits) + (size_t)b * a.ld;
  const int V = a.V;
  const float temp = a.temperature[b];
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;

  // max of scaled logits
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += SNT) mx = fmaxf(mx, ld_logit<T>(row, i) * inv_t);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = mx;
  if (threadIdx.x == 0) best = 0ull;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = sh[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) sh[34] = t;
  }
  __syncthreads();
  mx = sh[34];
  __syncthreads();

  float z = 0.f;
  for (int i = threadIdx.x; i < V; i += SNT) z += __expf(ld_logit<T>(row, i) * inv_t - mx);
  z = bsum<SNT>(z, sh);
  const float logz = logf(z);

  uint32_t cut = 0;  // keep keys >= cut
  if (greedy) {
    cut = f2key(0.f);  // only the max survives (ties -> lowest index below)
  } else {
    const int k = a.top_k ? a.top_k[b] : 0;
    if (k > 0 && k < V) cut = radix_cutoff<T>(row, V, inv_t, mx, 0, (float)k, 0u, hist, sh);
    const float p = a.top_p ? a.top_p[b] : 1.f;
    if (p < 1.f) {
      float zk = z;
      if (cut != 0) {
        float s = 0.f;
        for (int i = threadIdx.x; i < V; i += SNT) {
          const float x = ld_logit<T>(row, i) * inv_t - mx;
          if (f2key(x) >= cut) s += __expf(x);
        }
        zk = bsum<SNT>(s, sh);
      }
      const uint32_t cp = radix_cutoff<T>(row, V, inv_t, mx, 1, p * zk, cut, hist, sh);
      cut = max(cut, cp);
    }
  }

  // Gumbel-max draw among kept tokens; pack (score key, ~index) to take the
  // max score and, on ties, the lowest index.
  const uint32_t seed_lo = (uint32_t)a.rng[2 * b], seed_hi = (uint32_t)((uint64_t)a.rng[2 * b] >> 32);
  const uint64_t off = (uint64_t)a.rng[2 * b + 1];
  unsigned long long mine = 0ull;
  const int nwords = (V + 31) / 32;
  for (int base = 0; base < V; base += SNT) {
    const int i = base + threadIdx.x;
    bool keep = false;
    if (i < V) {
      const float x = ld_logit<T>(row, i) * inv_t - mx;
      keep = f2key(x) >= cut;
      if (keep) {
        float score = x;
        if (!greedy) {
          uint32_t c[4] = {(uint32_t)i, (uint32_t)b, (uint32_t)off, (uint32_t)(off >> 32)};
          philox4x32_10(c, seed_lo, seed_hi);
          const float u = ((float)c[0] + 0.5f) * 2.3283064365386963e-10f;
          score = x - logf(-logf(u));
        }
        const unsigned long long cand =
            ((unsigned long long)f2key(score) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
        if (cand > mine) mine = cand;
      }
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, keep);
    if (a.keep_mask && (threadIdx.x & 31) == 0) {
      const int w = (base + (threadIdx.x & ~31)) / 32;
      if (w < nwords) a.keep_mask[(size_t)b * nwords + w] = bal;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, mine, o);
    if (other > mine) mine = other;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(&best, mine);
  __syncthreads();
  if (threadIdx.x == 0) {
    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    a.out_tok[b] = tok;
    if (a.out_logprob) a.out_logprob[b] = ld_logit<T>(row, tok) * inv_t - mx - logz;
  }
}

// logit -> logit / penalty if > 0 else logit * penalty, for each distinct id in
// prev[b, :] (padded with -1). Restates openmini-server/src/model/inference/sampler.rs:175-219.
template <typename T>
__global__ void rep_penalty_kernel(T* logits, int ld, int V, const int* prev, int L, const float* penalty) {
  const int b = blockIdx.x;
  const float pen = penalty[b];
  if (pen == 1.f) return;
  T* row = logits + (size_t)b * ld;
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    const int id = prev[(size_t)b * L + j];
    if (id < 0 || id >= V) continue;
    bool first = true;  // apply once per distinct id
    for (int k = 0; k < j; ++k)
      if (prev[(size_t)b * L + k] == id) { first = false; break; }
    if (!first) continue;
    const float x = ld_logit<T>(row, id);
    const float y = x > 0.f ? x / pen : x * pen;
    if constexpr (std::is_same<T, float>::value) row[id] = y; else row[id] = __float2bfloat16_rn(y);
  }
}

}  // namespace om

void om_sample(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_p, torch::Tensor top_k,
               torch::Tensor rng, torch::Tensor out_tok, c10::optional<torch::Tensor> out_logprob,
               c10::optional<torch::Tensor> keep_mask) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "sample: logits [B, V]");
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  TORCH_CHECK(rng.scalar_type() == at::kLong && rng.numel() >= 2 * B && rng.is_contiguous(), "sample: rng int64 [B, 2]");
  TORCH_CHECK(temperature.scalar_type() == at::kFloat && top_p.scalar_type() == at::kFloat &&
                  top_k.scalar_type() == at::kInt,
              "sample: knob dtypes");
  om::SampleArgs a;
  a.logits = logits.data_ptr();
  a.ld = logits.stride(0);
  a.V = V;
  a.temperature = temperature.data_ptr<float>();
  a.top_p = top_p.data_ptr<float>();
  a.top_k = top_k.data_ptr<int>();
  a.rng = rng.data_ptr<int64_t>();
  a.out_tok = out_tok.data_ptr<int>();
  a.out_logprob = out_logprob.has_value() ? out_logprob->data_ptr<float>() : nullptr;
  a.keep_mask = nullptr;
  if (keep_mask.has_value()) {
    TORCH_CHECK(keep_mask->numel() >= (int64_t)B * ((V + 31) / 32), "sample: keep_mask too small");
    a.keep_mask = reinterpret_cast<uint32_t*>(keep_mask->data_ptr<int>());
  }
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (logits.scalar_type() == at::kFloat)
    om::sample_kernel<float><<<B, om::SNT, 0, st>>>(a);
  else if (logits.scalar_type() == at::kBFloat16)
    om::sample_kernel<__nv_bfloat16><<<B, om::SNT, 0, st>>>(a);
  else
    TORCH_CHECK(false, "sample: logits must be fp32 or bf16");
  OM_LAUNCH_CHECK();
}

void om_repetition_penalty(torch::Tensor logits, torch::Tensor prev, torch::Tensor penalty) {
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0 || prev.size(1) == 0) return;
  TORCH_CHECK(prev.scalar_type() == at::kInt && prev.is_contiguous(), "rep penalty: prev int32 [B, L]");
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (logits.scalar_type() == at::kFloat)
    om::rep_penalty_kernel<float><<<B, 256, 0, st>>>(logits.data_ptr<float>(), logits.stride(0), V,
                                                    prev.data_ptr<int>(), prev.size(1), penalty.data_ptr<float>());
  else
    om::rep_penalty_kernel<__nv_bfloat16><<<B, 256, 0, st>>>(
        reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V, prev.data_ptr<int>(),
        prev.size(1), penalty.data_ptr<float>());
  OM_LAUNCH_CHECK();
}
