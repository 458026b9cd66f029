// Symmetric peer memory (CUDA IPC over NVLink / NVSwitch) and the
// sequence-parallel collective kernels of the tensor-parallel decoder.
//
// Every rank allocates one buffer of the same size and maps every peer's
// buffer through CUDA IPC, so a kernel can load from and store to any rank's
// buffer with plain global loads / stores (peer-to-peer over NVLink 5). No
// multicast object and no TMA is involved.
//
// Buffer layout (identical on every rank):
//   [0, 256)    control words: ready[8] (offset 0), agdone[8] (offset 64),
//               epoch (offset 128), CTA ticket of sp_reduce (offset 132),
//               CTA ticket of the peer-output GEMM (offset 136)
//   [256, ...)  data regions addressed by byte offset (partials and gathered
//               activations, double-buffered by the caller)
//
// One all-reduce of the decoder (after o-proj / down-proj) becomes, with the
// residual stream sharded by token rows (rank r owns rows [r T/W, (r+1) T/W)):
//   sp_signal   epoch += 1; publish "my partial for this epoch is written"
//               (ready[me] = epoch on every peer, release at system scope)
//   sp_reduce   wait ready[p] >= epoch for all p; for each owned row: sum the W
//               partial rows read from the peers, add the residual row (updated
//               in place), RMSNorm, store the normed row into EVERY rank's
//               gather region (all-gather by push); the last CTA then bumps
//               agdone[me] on every peer
//   sp_wait     wait agdone[p] >= epoch for all p (the gathered activations are
//               complete); the next column-parallel GEMM reads them locally. A weight-only
//               decode GEMM does this wait itself (GemmArgs::agwait, in its activation
//               producer warp), so its weight stream starts before the gather completes.
// Pull mode (the default) folds sp_signal into sp_reduce (SpArgs::signal): block 0
// publishes ready[me] at the start and the last CTA stores the new epoch.
// so reduce-scatter, residual add, RMSNorm and all-gather are one kernel and
// each byte crosses NVLink once.
//
// Push variant (the default of the decoder): the row-parallel GEMM itself
// stores each output tile straight into the owner rank's partials slot
// ([world][rows_own][D], slot = source rank) as it leaves TMEM, and its last
// CTA publishes ready[me] = epoch on every rank (gemm_common.cuh PeerOut /
// peer_publish). The GEMM -> reduce-scatter is then one kernel whose NVLink
// transfer overlaps the remaining tiles' math, sp_signal is not launched, and
// sp_reduce (push = 1) sums the W slots from local memory. Every wait is bounded (OM_WAIT_LIMIT_NS) and
// records an error code instead of hanging.
//
// Reference counterpart: the tensor-parallel row split -> all_reduce and column
// split -> all_gather of openmini-server/src/distributed/tp.rs:506-625 over the
// CollectiveOps interface of distributed/communication.rs:85-177.
#include "../common/om_host.h"
#include "../common/om_ptx.cuh"

#include <cuda_bf16.h>

namespace om {

constexpr int SP_MAX_WORLD = 8;
constexpr int SP_CTRL_BYTES = 256;

struct SpArgs {
  uint8_t* base[SP_MAX_WORLD];  // every rank's buffer (own included)
  int rank, world;
  int rows_own;                 // rows owned by this rank (T / world)
  int D;
  long long p_off;              // partials region offset (-1: no reduction, normalise only)
  long long x_off;              // gathered normed-activation region offset
  int push;                     // 1: the partials were pushed into this rank's slots by the
                                // peer-output GEMM ([world][rows_own][D] at p_off, local reads)
  int signal;                   // 1: this kernel opens the epoch (epoch + 1) and block 0 publishes
                                // ready[rank] on every peer first (pull mode: the partials were
                                // written locally by the previous kernel)
  __nv_bfloat16* h;             // own residual rows [rows_own, D]
  const __nv_bfloat16* w;       // RMSNorm weight [D]
  float eps;
  int* status;
};

__device__ __forceinline__ int* ctrl(uint8_t* b, int off) { return reinterpret_cast<int*>(b + off); }

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until every peer's control word at `off` reached `target`.
__device__ bool sp_wait_all(const SpArgs& a, int off, int target, int code) {
  const uint64_t t0 = globaltimer();
  for (int p = 0; p < a.world; ++p) {
    const int* f = ctrl(a.base[a.rank], off) + p;
    uint32_t spins = 0;
    while (ld_acquire_sys(f) < target) {
      if ((++spins & 63u) == 0 && globaltimer() - t0 > OM_WAIT_LIMIT_NS) {
        record_error(a.status, code);
        return false;
      }
    }
  }
  return true;
}

__global__ void sp_signal_kernel(const __grid_constant__ SpArgs a) {
  if (threadIdx.x != 0) return;
  int* ep = ctrl(a.base[a.rank], 128);
  const int e = *ep + 1;
  *ep = e;
  __threadfence_system();  // the partials written by the previous kernels precede the flag
#pragma unroll
  for (int p = 0; p < SP_MAX_WORLD; ++p)
    if (p < a.world) st_release_sys(ctrl(a.base[p], 0) + a.rank, e);
}

template <int NT>
__global__ void __launch_bounds__(NT) sp_reduce_norm_gather_kernel(const __grid_constant__ SpArgs a) {
  __shared__ float red[NT / 32];
  __shared__ int go;
  // epoch of this event: pushed partials -> the GEMM already advanced it; signal mode ->
  // every CTA reads the previous value here and the last CTA stores e at the end (after
  // every CTA has taken its ticket, so no CTA can read the new value at its start)
  const int e = *ctrl(a.base[a.rank], 128) + (a.signal ? 1 : 0);
  if (a.signal && blockIdx.x == 0 && threadIdx.x == 0) {
    // the previous kernel's partials are complete (stream order); make them visible to the
    // peers before the flag they acquire
    __threadfence_system();
#pragma unroll
    for (int p = 0; p < SP_MAX_WORLD; ++p)
      if (p < a.world) st_release_sys(ctrl(a.base[p], 0) + a.rank, e);
  }
  // every event waits for every rank's signal, also without partials: a rank that signalled
  // has finished reading the gather region this event overwrites (it was two events ago)
  if (threadIdx.x == 0) go = sp_wait_all(a, 0, e, OM_ERR_WAIT_FULL) ? 1 : 0;
  __syncthreads();
  const int nv = a.D / 8;  // uint4 vectors per row
  if (go) {
    for (int r = blockIdx.x; r < a.rows_own; r += gridDim.x) {
      const size_t g = (size_t)a.rank * a.rows_own + r;  // global row
      __nv_bfloat16* hr = a.h + (size_t)r * a.D;
      float ss = 0.f;
      // pass 1: residual += sum of partials (rounded to bf16 as the residual stream), sum of squares
      for (int c = threadIdx.x; c < nv; c += NT) {
        float v[8];
        unpack8(reinterpret_cast<const uint4*>(hr)[c], v);
        if (a.p_off >= 0) {
          // issue every rank's load before the first add: the remote ones then overlap
          uint4 u[SP_MAX_WORLD];
#pragma unroll
          for (int p = 0; p < SP_MAX_WORLD; ++p) {
            if (p < a.world) {
              const uint8_t* src = a.push ? a.base[a.rank] + a.p_off + ((size_t)p * a.rows_own + r) * a.D * 2
                                          : a.base[p] + a.p_off + g * a.D * 2;
              u[p] = reinterpret_cast<const uint4*>(src)[c];
            }
          }
#pragma unroll
          for (int p = 0; p < SP_MAX_WORLD; ++p) {
            if (p < a.world) {
              float d[8];
              unpack8(u[p], d);
#pragma unroll
              for (int t = 0; t < 8; ++t) v[t] += d[t];
            }
          }
          const uint4 nu = pack8(v);
          reinterpret_cast<uint4*>(hr)[c] = nu;
          unpack8(nu, v);
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) ss += v[t] * v[t];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < NT / 32; ++i) tot += red[i];
      const float inv = rsqrtf(tot / a.D + a.eps);
      // pass 2: normalise and push the row into every rank's gather region
      for (int c = threadIdx.x; c < nv; c += NT) {
        float v[8], wf[8];
        unpack8(reinterpret_cast<const uint4*>(hr)[c], v);
        unpack8(reinterpret_cast<const uint4*>(a.w)[c], wf);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = v[t] * inv * wf[t];
        const uint4 o = pack8(v);
#pragma unroll
        for (int p = 0; p < SP_MAX_WORLD; ++p)
          if (p < a.world) reinterpret_cast<uint4*>(a.base[p] + a.x_off + g * a.D * 2)[c] = o;
      }
      __syncthreads();  // red[] reuse
    }
  }
  // publish: every thread fences its own peer stores, then the last CTA bumps agdone[me] everywhere
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* ticket = reinterpret_cast<unsigned*>(ctrl(a.base[a.rank], 132));
    const unsigned t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      *ticket = 0u;
      if (a.signal) *ctrl(a.base[a.rank], 128) = e;
      __threadfence_system();
#pragma unroll
      for (int p = 0; p < SP_MAX_WORLD; ++p)
        if (p < a.world) red_release_sys_add(ctrl(a.base[p], 64) + a.rank, 1);
    }
  }
}

__global__ void sp_wait_kernel(const __grid_constant__ SpArgs a) {
  if (threadIdx.x != 0) return;
  const int e = *ctrl(a.base[a.rank], 128);
  sp_wait_all(a, 64, e, OM_ERR_WAIT_FULL);
}

}  // namespace om

// ------------------------------------------------------------------ host side

int64_t om_symm_alloc(int64_t bytes) {
  void* p = nullptr;
  OM_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  OM_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  return reinterpret_cast<int64_t>(p);
}

void om_symm_free(int64_t ptr) { OM_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

torch::Tensor om_symm_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  OM_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::dtype(torch::kUInt8));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t om_symm_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.scalar_type() == at::kByte,
              "symm_open: handle bytes");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  OM_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void om_symm_close(int64_t ptr) { OM_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

// A tensor view of `bytes` at `ptr + offset` (no ownership).
torch::Tensor om_symm_view(int64_t ptr, int64_t offset, std::vector<int64_t> shape, int64_t dtype_code) {
  const auto dt = dtype_code == 0 ? torch::kBFloat16 : (dtype_code == 1 ? torch::kFloat : torch::kInt);
  int dev;
  OM_CUDA_CHECK(cudaGetDevice(&dev));
  return torch::from_blob(reinterpret_cast<uint8_t*>(ptr) + offset, shape,
                          torch::dtype(dt).device(torch::kCUDA, dev));
}

static om::SpArgs sp_args(const std::vector<int64_t>& bases, int64_t rank, int64_t rows_own, int64_t D,
                          int64_t p_off, int64_t x_off, torch::Tensor status) {
  TORCH_CHECK(!bases.empty() && bases.size() <= (size_t)om::SP_MAX_WORLD, "sp: 1..8 ranks");
  om::SpArgs a{};
  for (size_t i = 0; i < bases.size(); ++i) a.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  a.rank = rank;
  a.world = bases.size();
  a.rows_own = rows_own;
  a.D = D;
  a.p_off = p_off;
  a.x_off = x_off;
  a.status = status.data_ptr<int>();
  return a;
}

void om_sp_signal(std::vector<int64_t> bases, int64_t rank, torch::Tensor status) {
  om::SpArgs a = sp_args(bases, rank, 0, 8, -1, 0, status);
  om::sp_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream().stream()>>>(a);
  OM_LAUNCH_CHECK();
}

// h: own residual rows [rows_own, D] (updated in place when p_off >= 0);
// normed rows land at x_off + global_row * D * 2 of every rank's buffer.
void om_sp_reduce_norm_gather(std::vector<int64_t> bases, int64_t rank, torch::Tensor h, torch::Tensor w,
                              double eps, int64_t p_off, int64_t x_off, torch::Tensor status, bool push,
                              bool signal) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.dim() == 2, "sp_reduce: h");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.numel() == h.size(1), "sp_reduce: w");
  const int D = h.size(1);
  TORCH_CHECK(D % 8 == 0, "sp_reduce: D % 8");
  TORCH_CHECK((p_off < 0 || p_off % 16 == 0) && x_off % 16 == 0 && x_off >= om::SP_CTRL_BYTES, "sp_reduce: offsets");
  om::SpArgs a = sp_args(bases, rank, h.size(0), D, p_off, x_off, status);
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.eps = eps;
  a.push = push ? 1 : 0;
  a.signal = signal ? 1 : 0;
  TORCH_CHECK(!(push && signal), "sp_reduce: pushed partials come with their own signal");
  const int grid = std::max<int>(1, std::min<int>(a.rows_own, 2 * om::num_sms()));
  // one thread per 16-byte vector of the row (up to 1024): every partial row of every peer
  // is then requested at once, so a pulled row costs one NVLink round trip, not one per chunk
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (D / 8 >= 1024)
    om::sp_reduce_norm_gather_kernel<1024><<<grid, 1024, 0, st>>>(a);
  else if (D / 8 >= 512)
    om::sp_reduce_norm_gather_kernel<512><<<grid, 512, 0, st>>>(a);
  else
    om::sp_reduce_norm_gather_kernel<256><<<grid, 256, 0, st>>>(a);
  OM_LAUNCH_CHECK();
}

void om_sp_wait(std::vector<int64_t> bases, int64_t rank, torch::Tensor status) {
  om::SpArgs a = sp_args(bases, rank, 0, 8, -1, 0, status);
  om::sp_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream().stream()>>>(a);
  OM_LAUNCH_CHECK();
}
