// Token sampler: temperature -> top-k -> top-p -> draw.
//
// The reference sampler (openmini-server/src/model/inference/sampler.rs:220-450,
// openmini-server/src/model/inference/model.rs:3970) sorts the vocabulary. Here
// each row is handled by one thread-block cluster of SCL CTAs: every CTA keeps
// its slice of the row in registers, and the top-k / top-p cut-offs are found
// without sorting by a bitwise binary search over order-preserving keys of the
// logits (16-bit keys for bf16 logits, 32-bit for fp32): each probe is a plain
// count (top-k) or probability-mass (top-p) reduction, combined across the
// cluster through distributed shared memory. Top-p keeps the smallest
// descending prefix whose mass reaches p (ties at the cut-off are kept), over
// the top-k-restricted distribution. The draw is a Gumbel-max race among the
// kept tokens with Philox-4x32-10 counter-based uniforms (Salmon et al.,
// SC'11), so a (seed, offset) pair reproduces the draw exactly.
//
// Outputs: the token, its log-probability under the temperature-scaled full
// distribution, and optionally the kept set as a bitmask (bit i of word i/32)
// for sampling-mask replay in RL training.
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

namespace om {

constexpr int SCL = 8;    // CTAs per row (portable cluster size)
constexpr int SNT = 512;  // threads per CTA

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
  int ld, V, chunk;  // chunk: elements per CTA (multiple of 32)
  const float* temperature;
  const float* top_p;
  const int* top_k;
  const int64_t* rng;  // [B, 2] = (seed, offset)
  int* out_tok;
  float* out_logprob;
  uint32_t* keep_mask;  // [B, ceil(V/32)] or null
};

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_dsmem_u64(uint32_t addr) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
  return v;
}

struct SampleSmem {
  float warp_part[SNT / 32];
  float slot[2];                 // this CTA's partial, double-buffered by pass parity
  unsigned long long best_warp[SNT / 32];
  unsigned long long best;
};

// Sum of v over the cluster (op 0) or max (op 1); every thread gets the result.
__device__ __forceinline__ float cluster_reduce(float v, int op, SampleSmem& sm, int& pass) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = op ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sm.warp_part[warp] = v;
  __syncthreads();
  const int buf = pass & 1;
  if (warp == 0) {
    float t = lane < SNT / 32 ? sm.warp_part[lane] : (op ? -INFINITY : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, t, o);
      t = op ? fmaxf(t, w) : t + w;
    }
    if (lane == 0) sm.slot[buf] = t;
  }
  cluster_sync();
  const uint32_t a = smem_u32(&sm.slot[buf]);
  float r = op ? -INFINITY : 0.f;
#pragma unroll
  for (int c = 0; c < SCL; ++c) {
    const float w = ld_dsmem_f32(mapa(a, c));
    r = op ? fmaxf(r, w) : r + w;
  }
  ++pass;
  return r;
}

template <typename T, int EPT>
__global__ void __cluster_dims__(SCL, 1, 1) __launch_bounds__(SNT) sample_kernel(const SampleArgs a) {
  __shared__ SampleSmem sm;
  const int b = blockIdx.x / SCL;
  const uint32_t crank = cluster_rank();
  const T* row = reinterpret_cast<const T*>(a.logits) + (size_t)b * a.ld;
  const int V = a.V;
  const int base = (int)crank * a.chunk;
  const float temp = a.temperature[b];
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;
  constexpr int KEY_SHIFT = std::is_same<T, float>::value ? 0 : 16;
  constexpr int KEY_BITS = 32 - KEY_SHIFT;
  int pass = 0;

  float x[EPT];
  uint32_t key[EPT];
  float lmax = -INFINITY;
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    const int i = base + e * SNT + (int)threadIdx.x;
    const bool in = (e * SNT + (int)threadIdx.x) < a.chunk && i < V;
    const float l = in ? ld_logit<T>(row, i) : -INFINITY;
    x[e] = l * inv_t;
    key[e] = in ? (f2key(l) >> KEY_SHIFT) : 0u;  // key 0: never kept
    lmax = fmaxf(lmax, x[e]);
  }
  const float mx = cluster_reduce(lmax, 1, sm, pass);
  float z = 0.f;
#pragma unroll
  for (int e = 0; e < EPT; ++e) z += __expf(x[e] - mx);
  z = cluster_reduce(z, 0, sm, pass);

  uint32_t cut = 1;  // keep key >= cut (real keys are >= 1)
  if (greedy) {
    // keep only the maximum (ties broken toward the lowest index below)
    cut = 0xFFFFFFFFu;
#pragma unroll
    for (int e = 0; e < EPT; ++e)
      if (x[e] == mx && key[e] != 0u) cut = min(cut, key[e]);
    cut = (uint32_t)(-cluster_reduce(-(float)cut, 1, sm, pass));  // exact for 16-bit keys
    if (KEY_BITS == 32) {
      // fp32 keys may not survive the float round trip: fall back to comparing values
      cut = 0;
    }
  } else {
    const int k = a.top_k ? a.top_k[b] : 0;
    if (k > 0 && k < V) {
      uint32_t t = 0;
      for (int bit = KEY_BITS - 1; bit >= 0; --bit) {
        const uint32_t cand = t | (1u << bit);
        float c = 0.f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) c += key[e] >= cand ? 1.f : 0.f;
        if (cluster_reduce(c, 0, sm, pass) >= (float)k) t = cand;
      }
      cut = max(cut, t);
    }
    const float p = a.top_p ? a.top_p[b] : 1.f;
    if (p < 1.f) {
      float zk = z;
      if (cut > 1) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) s += key[e] >= cut ? __expf(x[e] - mx) : 0.f;
        zk = cluster_reduce(s, 0, sm, pass);
      }
      const float target = p * zk;
      uint32_t t = 0;
      for (int bit = KEY_BITS - 1; bit >= 0; --bit) {
        const uint32_t cand = t | (1u << bit);
        if (cand < cut) {  // below the top-k floor every probe passes
          t = cand;
          continue;
        }
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) s += key[e] >= cand ? __expf(x[e] - mx) : 0.f;
        if (cluster_reduce(s, 0, sm, pass) >= target) t = cand;
      }
      cut = max(cut, t);
    }
  }

  // Gumbel-max draw among kept tokens; pack (score key, ~index) so the max
  // picks the highest score and, on ties, the lowest index.
  const uint32_t seed_lo = (uint32_t)a.rng[2 * b], seed_hi = (uint32_t)((uint64_t)a.rng[2 * b] >> 32);
  const uint64_t off = (uint64_t)a.rng[2 * b + 1];
  unsigned long long mine = 0ull;
  const int nwords = (V + 31) / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    const int li = e * SNT + (int)threadIdx.x;
    const int i = base + li;
    bool keep = key[e] != 0u && (greedy && KEY_BITS == 32 ? x[e] == mx : key[e] >= cut);
    if (keep) {
      float score = x[e] - mx;
      if (!greedy) {
        // counter (token, 0, offset) under key = the request's seed: a draw depends on the
        // request's seed and step only, not on its row in the batch or the TP split
        uint32_t c[4] = {(uint32_t)i, 0u, (uint32_t)off, (uint32_t)(off >> 32)};
        philox4x32_10(c, seed_lo, seed_hi);
        const float u = ((float)c[0] + 0.5f) * 2.3283064365386963e-10f;
        score -= logf(-logf(u));
      }
      const unsigned long long cand =
          ((unsigned long long)f2key(score) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
      if (cand > mine) mine = cand;
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, keep);
    if (a.keep_mask && lane == 0 && li - lane < a.chunk) {
      const int w = (base + li - lane) / 32;
      if (w < nwords) a.keep_mask[(size_t)b * nwords + w] = bal;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, mine, o);
    if (other > mine) mine = other;
  }
  if (lane == 0) sm.best_warp[warp] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0ull;
    for (int w = 0; w < SNT / 32; ++w) m = sm.best_warp[w] > m ? sm.best_warp[w] : m;
    sm.best = m;
  }
  cluster_sync();
  if (crank == 0 && threadIdx.x == 0) {
    unsigned long long m = 0ull;
    const uint32_t addr = smem_u32(&sm.best);
    for (int c = 0; c < SCL; ++c) {
      const unsigned long long w = ld_dsmem_u64(mapa(addr, c));
      m = w > m ? w : m;
    }
    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFull));
    a.out_tok[b] = tok;
    if (a.out_logprob) a.out_logprob[b] = ld_logit<T>(row, tok) * inv_t - mx - logf(z);
  }
  cluster_sync();  // keep every CTA's shared memory alive until rank 0 has read it
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

template <typename T>
static void launch_sample(const SampleArgs& a, int B, cudaStream_t st) {
  const int ept = (a.chunk + SNT - 1) / SNT;
  if (ept <= 8)
    sample_kernel<T, 8><<<B * SCL, SNT, 0, st>>>(a);
  else if (ept <= 16)
    sample_kernel<T, 16><<<B * SCL, SNT, 0, st>>>(a);
  else if (ept <= 32)
    sample_kernel<T, 32><<<B * SCL, SNT, 0, st>>>(a);
  else if (ept <= 48)
    sample_kernel<T, 48><<<B * SCL, SNT, 0, st>>>(a);
  else
    TORCH_CHECK(false, "sample: vocabulary too large (max ", SCL * SNT * 48, ")");
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
  a.chunk = ((V + om::SCL - 1) / om::SCL + 31) / 32 * 32;
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
    om::launch_sample<float>(a, B, st);
  else if (logits.scalar_type() == at::kBFloat16)
    om::launch_sample<__nv_bfloat16>(a, B, st);
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
