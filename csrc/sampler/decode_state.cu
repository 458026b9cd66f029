// Device-side advance of the decode state between consecutive decode steps,
// so several decode steps can be replayed back to back from a CUDA graph with
// no host round trip (multi-step decoding). For each live row b:
//   ids[b] = sampled[b]; pos[b] += 1; ctx[b] += 1; rng offset += 1
//   slot[b] = block_table[b][pos / 16] * 16 + pos % 16
//   hist[step * B + b] = sampled[b]        (step read from *step, then bumped)
// Rows with slot < 0 are padding and stay untouched.
#include "../common/om_host.h"

namespace om {

__global__ void decode_advance_kernel(const int* __restrict__ sampled, int* ids, int* pos, int* ctx, int* slots,
                                      const int* __restrict__ bt, int mb, int64_t* rng, int* hist, int* step,
                                      int B, int hist_steps) {
  const int b = threadIdx.x;
  const int s = *step;
  __syncthreads();
  if (b < B && slots[b] >= 0) {
    const int t = sampled[b];
    ids[b] = t;
    const int p = pos[b] + 1;
    pos[b] = p;
    ctx[b] = ctx[b] + 1;
    const int bi = min(p >> 4, mb - 1);
    slots[b] = bt[(size_t)b * mb + bi] * 16 + (p & 15);
    rng[2 * b + 1] += 1;
    if (hist && s < hist_steps) hist[(size_t)s * B + b] = t;
  }
  __syncthreads();
  if (b == 0) *step = s + 1;
}

}  // namespace om

void om_decode_advance(torch::Tensor sampled, torch::Tensor ids, torch::Tensor pos, torch::Tensor ctx,
                       torch::Tensor slots, torch::Tensor bt, torch::Tensor rng, c10::optional<torch::Tensor> hist,
                       torch::Tensor step) {
  const int B = ids.numel();
  TORCH_CHECK(B <= 1024, "decode_advance: at most 1024 rows");
  TORCH_CHECK(bt.stride(1) == 1 && bt.size(0) >= B, "decode_advance: block table");
  auto st = at::cuda::getCurrentCUDAStream().stream();
  int* hp = nullptr;
  int hs = 0;
  if (hist.has_value()) {
    hp = hist->data_ptr<int>();
    hs = hist->numel() / std::max(B, 1);
  }
  om::decode_advance_kernel<<<1, 1024, 0, st>>>(sampled.data_ptr<int>(), ids.data_ptr<int>(), pos.data_ptr<int>(),
                                                ctx.data_ptr<int>(), slots.data_ptr<int>(), bt.data_ptr<int>(),
                                                bt.stride(0), rng.data_ptr<int64_t>(), hp, step.data_ptr<int>(), B,
                                                hs);
  OM_LAUNCH_CHECK();
}
