// Token sampler: temperature -> top-k -> top-p -> draw.
//
// The reference sampler (openmini-server/src/model/inference/sampler.rs:220-450,
// openmini-server/src/model/inference/model.rs:3970) sorts the vocabulary. Here
// each row is handled by one thread-block cluster of SCL CTAs: every CTA keeps
// its slice of the row in registers, and the top-k / top-p cut-offs are found
// without sorting by a radix search over order-preserving keys of the logits
// (16-bit keys for bf16 logits, 32-bit for fp32), 2 bits per pass: each pass
// evaluates the 3 candidates of the next digit at once as count (top-k) or
// probability-mass (top-p) sums over precomputed probabilities, combined across
// the cluster through distributed shared memory in one exchange. Top-p keeps the smallest
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
  int row0;             // global index of row 0 (row-parallel sampling under TP): the draw of
                        // row b uses counter row0 + b, so it does not depend on the split
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
  float vec_part[SNT / 32][16];  // cluster_reduce_vec: per-warp partials
  float vec_slot[2][16];         // this CTA's partials, double-buffered by pass parity
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

// Sums of NV values over the cluster (every thread passes its NV partials and gets
// the NV totals): one CTA-wide and one cluster-wide exchange for all NV values.
template <int NV>
__device__ __forceinline__ void cluster_reduce_vec(float (&v)[NV], float (*warp_part)[16], float (*slot)[16],
                                                   int& pass) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < NV; ++i) warp_part[warp][i] = v[i];
  __syncthreads();
  const int buf = pass & 1;
  if (threadIdx.x < NV) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < SNT / 32; ++w) t += warp_part[w][threadIdx.x];
    slot[buf][threadIdx.x] = t;
  }
  cluster_sync();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t a = smem_u32(&slot[buf][i]);
    float r = 0.f;
#pragma unroll
    for (int c = 0; c < SCL; ++c) r += ld_dsmem_f32(mapa(a, c));
    v[i] = r;
  }
  ++pass;
}

// Largest key threshold t with S(t) >= target, where S(t) = sum of w over the
// elements whose key >= t (monotone non-increasing in t), searched DB bits per
// pass: each pass evaluates the 2^DB - 1 candidates of the next digit at once, so
// a 16-bit search takes 16 / DB cluster reductions. `floor` is a lower bound
// already known to satisfy the predicate.
template <int EPT, int KEY_BITS, bool MASS, int DB>
__device__ __forceinline__ uint32_t search_cut(const uint32_t (&key)[EPT], const float (&p)[EPT], float target,
                                               uint32_t floor, float (*warp_part)[16], float (*slot)[16],
                                               int& pass) {
  constexpr int NC = (1 << DB) - 1;
  uint32_t t = 0;
  for (int sh = KEY_BITS - DB; sh >= 0; sh -= DB) {
    float s[NC];
#pragma unroll
    for (int d = 0; d < NC; ++d) s[d] = 0.f;
    const uint32_t hi = t >> sh;  // decided prefix (digit position zero)
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const uint32_t kh = key[e] >> sh;
      // digit of the key relative to the prefix: below (none), inside, above (all)
      const int dg = kh < hi ? -1 : (kh - hi > (uint32_t)NC ? NC : (int)(kh - hi));
      const float w = MASS ? p[e] : 1.f;
#pragma unroll
      for (int d = 0; d < NC; ++d) s[d] += dg >= d + 1 ? w : 0.f;
    }
    cluster_reduce_vec<NC>(s, warp_part, slot, pass);
    int best = 0;
#pragma unroll
    for (int d = 0; d < NC; ++d)
      if (s[d] >= target || (t | ((uint32_t)(d + 1) << sh)) <= floor) best = d + 1;
    t |= (uint32_t)best << sh;
  }
  return t;
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
  float p[EPT];  // unnormalised probabilities exp(x - mx)
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    p[e] = __expf(x[e] - mx);
    z += p[e];
  }
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
    if (k > 0 && k < V) cut = max(cut, search_cut<EPT, KEY_BITS, false, 2>(key, p, (float)k, 0u, sm.vec_part,
                                                                         sm.vec_slot, pass));
    const float tp = a.top_p ? a.top_p[b] : 1.f;
    if (tp < 1.f) {
      float zk = z;
      if (cut > 1) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) s += key[e] >= cut ? p[e] : 0.f;
        zk = cluster_reduce(s, 0, sm, pass);
      }
      // below the top-k floor every probe passes (the mass there is at least zk)
      cut = max(cut, search_cut<EPT, KEY_BITS, true, 2>(key, p, tp * zk, cut, sm.vec_part, sm.vec_slot, pass));
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
    // (the scaled logit is re-read here rather than kept live through the cut-off search)
    const float xe = key[e] != 0u ? ld_logit<T>(row, i) * inv_t : -INFINITY;
    bool keep = key[e] != 0u && (greedy && KEY_BITS == 32 ? xe == mx : key[e] >= cut);
    if (keep) {
      float score = xe - mx;
      if (!greedy) {
        uint32_t c[4] = {(uint32_t)i, (uint32_t)(a.row0 + b), (uint32_t)off, (uint32_t)(off >> 32)};
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
               c10::optional<torch::Tensor> keep_mask, int64_t row0) {
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
  a.row0 = (int)row0;
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
