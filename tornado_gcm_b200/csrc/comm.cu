// Fused gradient all-reduce over NVLink peer memory (sm_100a).
//
// Every rank's fp32 gradient buffer lives in symmetric memory, so each rank
// holds device pointers to all peers' buffers and signal pads.  One kernel
// does the whole mean all-reduce ("two-shot" in one launch):
//
//   phase 0  per-block barrier: block b of every rank announces, in every
//            peer's signal pad, that its gradients are ready (the kernel runs
//            after backward on the rank's stream);
//   phase 1  reduce-scatter + all-gather: rank r owns chunk r; block b of
//            rank r reads its slice of chunk r from all W peers (16-byte P2P
//            loads), sums, multiplies by 1/W (the averaging, fused) and writes
//            the result into chunk r of every peer (P2P stores);
//   phase 2  per-block barrier, so that no rank uses its buffer before every
//            peer's pushes into it have landed.
//
// Signals are epoch counters (uint32) in the pads: pad[phase][src_rank][block]
// (2 x 8 x blocks words per rank, zeroed once at set-up).
// A block's epoch is one more than the value it last wrote, so no host value
// is baked into a captured CUDA graph.  Every wait is bounded (1 s of
// %globaltimer): on expiry the kernel records an error code in `err` and the
// block returns; the host reads the flag.  No TMA and no multicast is used:
// peer memory is touched only with plain loads and stores.

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <cstdint>

namespace tgcm {
namespace {

constexpr int kArThreads = 512;
constexpr int kArMaxRanks = 8;
constexpr uint64_t kArWaitNs = 1000000000ull;
constexpr int kErrArTimeout = 20;

__device__ __forceinline__ uint64_t ar_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ArArgs {
  float* bufs[kArMaxRanks];        // peers' gradient buffers (index = rank)
  uint32_t* pads[kArMaxRanks];     // peers' signal pads
  long long n;                     // elements per buffer
  int world, rank, blocks;
  float scale;
  int* err;
};

// Block-level barrier on `phase`: announce `epoch` to every peer, then wait
// until every peer announced it to us.  Returns false on timeout.
__device__ bool ar_barrier(const ArArgs& a, int phase, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x < a.world) {
    const int p = threadIdx.x;
    __threadfence_system();
    st_release_sys(a.pads[p] + (phase * kArMaxRanks + a.rank) * a.blocks + blockIdx.x, epoch);
  }
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint32_t* slot = a.pads[a.rank] + (phase * kArMaxRanks + threadIdx.x) * a.blocks + blockIdx.x;
    const uint64_t t0 = ar_now();
    while (static_cast<int32_t>(ld_acquire_sys(slot) - epoch) < 0) {
      if (ar_now() - t0 > kArWaitNs) {
        if (a.err) atomicCAS(a.err, 0, kErrArTimeout);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(kArThreads) fused_allreduce_kernel(ArArgs a) {
  // epoch: one more than what this block last announced for phase 0 on its own pad
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0)
    s_epoch = *(volatile uint32_t*)(a.pads[a.rank] + (0 * kArMaxRanks + a.rank) * a.blocks + blockIdx.x) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (!ar_barrier(a, 0, epoch)) return;

  // this rank's chunk, split over the blocks in 16-byte vectors
  const long long chunk = (a.n + a.world - 1) / a.world;
  const long long c0 = static_cast<long long>(a.rank) * chunk;
  long long c1 = c0 + chunk;
  if (c1 > a.n) c1 = a.n;
  const long long per = ((c1 - c0 + a.blocks - 1) / a.blocks + 3) / 4 * 4;
  const long long b0 = c0 + per * blockIdx.x;
  long long b1 = b0 + per;
  if (b1 > c1) b1 = c1;
  if (b0 < b1) {
    const bool vec = (b0 % 4 == 0);
    const long long nv = vec ? (b1 - b0) / 4 : 0;
    for (long long i = threadIdx.x; i < nv; i += blockDim.x) {
      const long long e = b0 + 4 * i;
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < a.world; ++p) {
        const float4 v = __ldcv(reinterpret_cast<const float4*>(a.bufs[p] + e));
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
      s.x *= a.scale; s.y *= a.scale; s.z *= a.scale; s.w *= a.scale;
      for (int p = 0; p < a.world; ++p) *reinterpret_cast<float4*>(a.bufs[p] + e) = s;
    }
    for (long long e = b0 + 4 * nv + threadIdx.x; e < b1; e += blockDim.x) {
      float s = 0.f;
      for (int p = 0; p < a.world; ++p) s += __ldcv(a.bufs[p] + e);
      s *= a.scale;
      for (int p = 0; p < a.world; ++p) a.bufs[p][e] = s;
    }
  }
  ar_barrier(a, 1, epoch);
}

// The two halves of the sharded-optimizer step (gradients and AdamW state
// split over the ranks by flat chunk; chunk r of the flat buffers belongs to
// rank r, the buffers hold a multiple of 4 * world elements):
//
//   fused_reduce_scatter_kernel  barrier on pad phase 0, then rank r sums
//       chunk r of every peer's gradient buffer (16-byte peer loads), scales
//       it and stores it into its OWN buffer only; nothing is pushed.
//   fused_all_gather_kernel      barrier on pad phase 1 (every rank's
//       optimizer has updated its chunk of the parameters), then rank r pulls
//       chunk p of the parameters from every peer p into its own buffer.
//
// Neither needs a closing barrier: a peer overwrites its gradient buffer only
// when it zeroes it for the next step, which follows its own all-gather and
// therefore our arrival at phase 1; it overwrites its parameter chunk only in
// its next optimizer step, which follows its next reduce-scatter and
// therefore our arrival at the next phase 0.  Each kernel keeps its own
// epoch on its own phase of the pad.
__device__ __forceinline__ void chunk_block_range(const ArArgs& a, int owner, long long& b0, long long& b1) {
  const long long chunk = a.n / a.world;
  const long long c0 = static_cast<long long>(owner) * chunk;
  const long long per = ((chunk + a.blocks - 1) / a.blocks + 3) / 4 * 4;
  b0 = c0 + per * blockIdx.x;
  b1 = b0 + per;
  if (b1 > c0 + chunk) b1 = c0 + chunk;
}

__global__ void __launch_bounds__(kArThreads) fused_reduce_scatter_kernel(ArArgs a) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0)
    s_epoch = *(volatile uint32_t*)(a.pads[a.rank] + (0 * kArMaxRanks + a.rank) * a.blocks + blockIdx.x) + 1u;
  __syncthreads();
  if (!ar_barrier(a, 0, s_epoch)) return;
  long long b0, b1;
  chunk_block_range(a, a.rank, b0, b1);
  float* dst = a.bufs[a.rank];
  for (long long e = b0 + 4 * threadIdx.x; e < b1; e += 4 * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < a.world; ++q) {
      const int p = (a.rank + q) % a.world;  // staggered: ranks start on different peers
      const float4 v = __ldcv(reinterpret_cast<const float4*>(a.bufs[p] + e));
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    s.x *= a.scale; s.y *= a.scale; s.z *= a.scale; s.w *= a.scale;
    *reinterpret_cast<float4*>(dst + e) = s;
  }
}

__global__ void __launch_bounds__(kArThreads) fused_all_gather_kernel(ArArgs a) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0)
    s_epoch = *(volatile uint32_t*)(a.pads[a.rank] + (1 * kArMaxRanks + a.rank) * a.blocks + blockIdx.x) + 1u;
  __syncthreads();
  if (!ar_barrier(a, 1, s_epoch)) return;
  float* dst = a.bufs[a.rank];
  for (int q = 1; q < a.world; ++q) {
    const int p = (a.rank + q) % a.world;
    long long b0, b1;
    chunk_block_range(a, p, b0, b1);
    const float* src = a.bufs[p];
    for (long long e = b0 + 4 * threadIdx.x; e < b1; e += 4 * blockDim.x)
      *reinterpret_cast<float4*>(dst + e) = __ldcv(reinterpret_cast<const float4*>(src + e));
  }
}

// Pull copy of static peer buffers: dst[p * bytes + i] = src_p[i] for every
// rank p (its own buffer included), 16-byte plain loads over NVLink.  Used
// for weight shards that do not change after set-up, so no barrier is needed.
struct PullArgs {
  const uint4* src[kArMaxRanks];
  uint4* dst;
  long long vecs;  // 16-byte vectors per source
  int world;
};

__global__ void __launch_bounds__(256) pull_peer_buffers_kernel(PullArgs a) {
  const long long total = a.vecs * a.world;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(i / a.vecs);
    a.dst[i] = a.src[p][i - p * a.vecs];
  }
}

// Stand-alone cross-rank barrier on a signal pad (one block): every rank
// announces the next epoch in every peer's pad and waits (bounded) for all
// peers' announcements.  Orders the peer reductions of a preceding kernel
// (fused Legendre analysis) before the ranks read their buffers.
__global__ void __launch_bounds__(32) peer_barrier_kernel(ArArgs a) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = *(volatile uint32_t*)(a.pads[a.rank] + a.rank) + 1u;
  __syncthreads();
  ar_barrier(a, 0, s_epoch);
}

}  // namespace

// pad_ptrs: int64 (world) CPU tensor of the peers' signal pads (>= 2 * 8 words each, zeroed once)
void peer_barrier(const at::Tensor& pad_ptrs, int64_t rank, const c10::optional<at::Tensor>& err, int64_t device) {
  TORCH_CHECK(pad_ptrs.scalar_type() == at::kLong && !pad_ptrs.is_cuda(), "pad_ptrs must be an int64 CPU tensor");
  const int64_t world = pad_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= kArMaxRanks && rank >= 0 && rank < world, "1..8 ranks supported");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  ArArgs a;
  memset(&a, 0, sizeof(a));
  for (int64_t p = 0; p < world; ++p) a.pads[p] = reinterpret_cast<uint32_t*>(pad_ptrs.data_ptr<int64_t>()[p]);
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.blocks = 1;
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  peer_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// buf: this rank's symmetric fp32 buffer; buf_ptrs / pad_ptrs: int64 (world)
// host tensors of the peers' buffer and signal-pad addresses.  The sum is
// multiplied by `scale`; 0 selects 1/world (the mean).
void fused_allreduce_mean(at::Tensor& buf, const at::Tensor& buf_ptrs, const at::Tensor& pad_ptrs, int64_t rank,
                          int64_t blocks, const c10::optional<at::Tensor>& err, double scale) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && buf.is_contiguous(), "fp32 CUDA buffer expected");
  TORCH_CHECK(buf_ptrs.scalar_type() == at::kLong && pad_ptrs.scalar_type() == at::kLong && !buf_ptrs.is_cuda() &&
                  !pad_ptrs.is_cuda(),
              "pointer tables must be int64 CPU tensors");
  const int64_t world = buf_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= kArMaxRanks && pad_ptrs.numel() == world, "1..8 ranks supported");
  TORCH_CHECK(blocks >= 1 && blocks <= 1024, "blocks out of range");
  c10::cuda::CUDAGuard guard(buf.device());
  ArArgs a;
  memset(&a, 0, sizeof(a));
  for (int64_t p = 0; p < world; ++p) {
    a.bufs[p] = reinterpret_cast<float*>(buf_ptrs.data_ptr<int64_t>()[p]);
    a.pads[p] = reinterpret_cast<uint32_t*>(pad_ptrs.data_ptr<int64_t>()[p]);
  }
  TORCH_CHECK(a.bufs[rank] == buf.data_ptr<float>(), "buffer is not this rank's symmetric allocation");
  a.n = buf.numel();
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.blocks = static_cast<int>(blocks);
  a.scale = scale == 0.0 ? 1.f / static_cast<float>(world) : static_cast<float>(scale);
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  fused_allreduce_kernel<<<static_cast<unsigned>(blocks), kArThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static ArArgs chunked_args(const at::Tensor& buf, const at::Tensor& buf_ptrs, const at::Tensor& pad_ptrs,
                           int64_t rank, int64_t blocks, const c10::optional<at::Tensor>& err, const char* what) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && buf.is_contiguous(), what,
              ": fp32 CUDA buffer expected");
  TORCH_CHECK(buf_ptrs.scalar_type() == at::kLong && pad_ptrs.scalar_type() == at::kLong && !buf_ptrs.is_cuda() &&
                  !pad_ptrs.is_cuda(),
              what, ": pointer tables must be int64 CPU tensors");
  const int64_t world = buf_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= kArMaxRanks && pad_ptrs.numel() == world && rank >= 0 && rank < world, what,
              ": 1..8 ranks supported");
  TORCH_CHECK(blocks >= 1 && blocks <= 1024, what, ": blocks out of range");
  TORCH_CHECK(buf.numel() % (4 * world) == 0, what, ": the buffer must hold a multiple of 4 * world elements");
  ArArgs a;
  memset(&a, 0, sizeof(a));
  for (int64_t p = 0; p < world; ++p) {
    a.bufs[p] = reinterpret_cast<float*>(buf_ptrs.data_ptr<int64_t>()[p]);
    a.pads[p] = reinterpret_cast<uint32_t*>(pad_ptrs.data_ptr<int64_t>()[p]);
  }
  TORCH_CHECK(a.bufs[rank] == buf.data_ptr<float>(), what, ": buffer is not this rank's symmetric allocation");
  for (int64_t p = 0; p < world; ++p)
    TORCH_CHECK(reinterpret_cast<uintptr_t>(a.bufs[p]) % 16 == 0, what, ": peer buffers must be 16-byte aligned");
  a.n = buf.numel();
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.blocks = static_cast<int>(blocks);
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  return a;
}

// In place: chunk `rank` of this rank's buffer becomes scale * (sum over the
// ranks of their chunk `rank`); the other chunks are left as they are.
// scale 0 selects 1/world.  pad_ptrs: signal pads of >= 2 * 8 * blocks words.
void fused_reduce_scatter(at::Tensor& buf, const at::Tensor& buf_ptrs, const at::Tensor& pad_ptrs, int64_t rank,
                          int64_t blocks, const c10::optional<at::Tensor>& err, double scale) {
  ArArgs a = chunked_args(buf, buf_ptrs, pad_ptrs, rank, blocks, err, "fused_reduce_scatter");
  a.scale = scale == 0.0 ? 1.f / static_cast<float>(a.world) : static_cast<float>(scale);
  c10::cuda::CUDAGuard guard(buf.device());
  fused_reduce_scatter_kernel<<<static_cast<unsigned>(blocks), kArThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// In place: chunk p of this rank's buffer is replaced by chunk p of rank p's
// buffer, for every p != rank.
void fused_all_gather(at::Tensor& buf, const at::Tensor& buf_ptrs, const at::Tensor& pad_ptrs, int64_t rank,
                      int64_t blocks, const c10::optional<at::Tensor>& err) {
  ArArgs a = chunked_args(buf, buf_ptrs, pad_ptrs, rank, blocks, err, "fused_all_gather");
  a.scale = 1.f;
  c10::cuda::CUDAGuard guard(buf.device());
  fused_all_gather_kernel<<<static_cast<unsigned>(blocks), kArThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dst (CUDA, contiguous, >= world * bytes_per_src bytes): the concatenation of the
// first bytes_per_src bytes of every peer buffer in src_ptrs (int64 CPU tensor).
void pull_peer_buffers(at::Tensor& dst, const at::Tensor& src_ptrs, int64_t bytes_per_src) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous(), "pull_peer_buffers: contiguous CUDA destination expected");
  TORCH_CHECK(src_ptrs.scalar_type() == at::kLong && !src_ptrs.is_cuda(), "src_ptrs must be an int64 CPU tensor");
  const int64_t world = src_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= kArMaxRanks, "1..8 sources supported");
  TORCH_CHECK(bytes_per_src > 0 && bytes_per_src % 16 == 0, "bytes_per_src must be a positive multiple of 16");
  TORCH_CHECK(dst.numel() * dst.element_size() >= world * bytes_per_src, "destination too small");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0, "destination must be 16-byte aligned");
  PullArgs a;
  memset(&a, 0, sizeof(a));
  for (int64_t p = 0; p < world; ++p) {
    const int64_t v = src_ptrs.data_ptr<int64_t>()[p];
    TORCH_CHECK(v % 16 == 0, "source buffers must be 16-byte aligned");
    a.src[p] = reinterpret_cast<const uint4*>(v);
  }
  a.dst = reinterpret_cast<uint4*>(dst.data_ptr());
  a.vecs = bytes_per_src / 16;
  a.world = static_cast<int>(world);
  c10::cuda::CUDAGuard guard(dst.device());
  const long long total = a.vecs * world;
  const unsigned blocks = static_cast<unsigned>(std::min<long long>((total + 255) / 256, 148LL * 4));
  pull_peer_buffers_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

namespace {

// out[i, l] = sum_w slots[w][i, l] for l < L (slots: W blocks of rows x ld floats);
// rows whose local row (i % period) is not valid are written as zeros (nobody
// stores into them, so the slots may hold a previous call's data there).
__global__ void slot_sum_kernel(const float* __restrict__ slots, float* __restrict__ out, int W, long long rows,
                                int ld, int L, long long slot_stride, const int* __restrict__ valid, int period) {
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long n = rows * L;
  if (idx >= n) return;
  const long long r = idx / L;
  const int l = static_cast<int>(idx - r * L);
  if (valid != nullptr && !__ldg(valid + r % period)) {
    out[idx] = 0.f;
    return;
  }
  const float* src = slots + r * ld + l;
  float s = 0.f;
  for (int w = 0; w < W; ++w) s += __ldg(src + w * slot_stride);
  out[idx] = s;
}

}  // namespace

// The owner's side of the sharded analysis: every rank stored its partial
// Legendre sums into its own slot of the owner's buffer (plain peer stores);
// after the barrier the owner adds the W slots.  slots: (W, rows, ld) fp32
// contiguous; returns (rows, L).
at::Tensor slot_sum(const at::Tensor& slots, int64_t W, int64_t rows, int64_t ld, int64_t L,
                    const c10::optional<at::Tensor>& valid) {
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == at::kFloat && slots.is_contiguous() &&
                  slots.numel() >= W * rows * ld && L <= ld && W >= 1,
              "slot_sum: contiguous fp32 (W, rows, ld) slots expected");
  c10::cuda::CUDAGuard guard(slots.device());
  const int* vp = nullptr;
  int period = 1;
  if (valid.has_value() && valid->defined()) {
    TORCH_CHECK(valid->is_cuda() && valid->scalar_type() == at::kInt && valid->is_contiguous() &&
                    valid->numel() >= 1 && rows % valid->numel() == 0,
                "slot_sum: valid must be an int32 CUDA vector whose length divides rows");
    vp = valid->data_ptr<int>();
    period = static_cast<int>(valid->numel());
  }
  auto out = at::empty({rows, L}, slots.options());
  const long long n = rows * L;
  if (n == 0) return out;
  slot_sum_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      slots.data_ptr<float>(), out.data_ptr<float>(), static_cast<int>(W), rows, static_cast<int>(ld),
      static_cast<int>(L), rows * ld, vp, period);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("slot_sum(Tensor slots, int W, int rows, int ld, int L, Tensor? valid=None) -> Tensor");
  m.def("fused_allreduce_mean(Tensor(a!) buf, Tensor buf_ptrs, Tensor pad_ptrs, int rank, int blocks, Tensor? err, float scale=0.0) -> ()");
  m.def("fused_reduce_scatter(Tensor(a!) buf, Tensor buf_ptrs, Tensor pad_ptrs, int rank, int blocks, Tensor? err, float scale=0.0) -> ()");
  m.def("fused_all_gather(Tensor(a!) buf, Tensor buf_ptrs, Tensor pad_ptrs, int rank, int blocks, Tensor? err) -> ()");
  m.def("pull_peer_buffers(Tensor(a!) dst, Tensor src_ptrs, int bytes_per_src) -> ()");
  m.def("peer_barrier(Tensor pad_ptrs, int rank, Tensor? err, int device) -> ()", &tgcm::peer_barrier);
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) {
  m.impl("fused_allreduce_mean", &tgcm::fused_allreduce_mean);
  m.impl("slot_sum", &tgcm::slot_sum);
  m.impl("fused_reduce_scatter", &tgcm::fused_reduce_scatter);
  m.impl("fused_all_gather", &tgcm::fused_all_gather);
  m.impl("pull_peer_buffers", &tgcm::pull_peer_buffers);
}
