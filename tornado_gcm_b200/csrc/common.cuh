// Shared device helpers for the sm_100a kernels: bounded mbarrier waits,
// TMA, tcgen05 (UMMA + TMEM) wrappers and the device error flag.
//
// Every wait on an mbarrier is bounded by a wall-clock budget read from
// %globaltimer.  On expiry the waiting thread records an error code in the
// caller-supplied device flag and returns false; callers then skip the rest
// of their work, wait (again bounded) for their own outstanding async
// operations and release TMEM, so a kernel never hangs the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace tgcm {

// Budget for one mbarrier wait (nanoseconds).  ~1 s: far above any
// legitimate wait in these kernels, short enough to keep the context alive.
constexpr uint64_t kWaitBudgetNs = 1000000000ull;

enum ErrorCode : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,
  kErrTimeoutEmpty = 2,
  kErrTimeoutTmemFull = 3,
  kErrTimeoutDrain = 4,
  kErrBounds = 5,
};

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* flag, int code) {
  if (flag != nullptr) atomicCAS(flag, 0, code);
}

// ── mbarrier ────────────────────────────────────────────────────────────────
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; returns false (and records `code`) when the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (global_timer_ns() - t0 > kWaitBudgetNs) {
      record_error(err, code);
      return false;
    }
  }
}

// ── TMA ─────────────────────────────────────────────────────────────────────
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled load (no multicast) completing on `bar` with byte accounting.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
      "r"(c2)
      : "memory");
}

// ── tcgen05 / TMEM ──────────────────────────────────────────────────────────
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Completion of all prior tcgen05 async ops of this thread arrives on `bar`.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::tf32 (fp32 operands read as TF32).
__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A * B, kind::f16 with BF16 operands (both A and B BF16).
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout.
// lbo/sbo in bytes; version bits = 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Shared-memory descriptor for an MN-major 32-bit (TF32) operand: 128-byte
// rows along MN with 32-byte swizzle atoms (layout type 1, the pattern the
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B: 32-byte chunk index
// XOR (row mod 4)).  lbo = bytes between 128-byte MN chunks, sbo = bytes
// between groups of 4 K-rows.
__device__ __forceinline__ uint64_t make_sw128b32_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 1ull << 61;
  return d;
}

// Instruction descriptor: f32 accumulate; fmt 1 = BF16, 2 = TF32;
// major 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t fmt, uint32_t a_major, uint32_t b_major, uint32_t M,
                                                  uint32_t N) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_major << 15) | (b_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// ── small math ──────────────────────────────────────────────────────────────
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ float gelu_tanh_grad_f(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  float u = k0 * (x + k1 * x * x * x);
  float t = tanhf(u);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

__device__ __forceinline__ float gelu_erf_f(float x) { return 0.5f * x * (1.f + erff(x * 0.7071067811865476f)); }

__device__ __forceinline__ float gelu_erf_grad_f(float x) {
  return 0.5f * (1.f + erff(x * 0.7071067811865476f)) + x * 0.3989422804014327f * expf(-0.5f * x * x);
}

enum Activation : int { kActNone = 0, kActRelu = 1, kActGelu = 2, kActGeluTanh = 3, kActSilu = 4, kActTanh = 5 };

// Hardware tanh (MUFU, relative error about 2^-11): used by the BF16 GEMM
// epilogues, whose outputs are rounded to BF16 (8-bit mantissa) anyway.
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh_hw(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.f + tanh_hw(u));
}

__device__ __forceinline__ float gelu_tanh_grad_hw(float x) {
  const float x2 = x * x;
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x2, x);
  const float t = tanh_hw(u);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * 0.7978845608028654f * fmaf(3.f * 0.044715f, x2, 1.f);
}

template <int ACT>
__device__ __forceinline__ float act_fast(float x) {
  if constexpr (ACT == kActRelu) return x > 0.f ? x : 0.f;
  else if constexpr (ACT == kActGelu) return gelu_erf_f(x);
  else if constexpr (ACT == kActGeluTanh) return gelu_tanh_hw(x);
  else if constexpr (ACT == kActSilu) return x / (1.f + __expf(-x));
  else if constexpr (ACT == kActTanh) return tanh_hw(x);
  else return x;
}

template <int ACT>
__device__ __forceinline__ float act_grad_fast(float x) {
  if constexpr (ACT == kActRelu) return x > 0.f ? 1.f : 0.f;
  else if constexpr (ACT == kActGelu) return gelu_erf_grad_f(x);
  else if constexpr (ACT == kActGeluTanh) return gelu_tanh_grad_hw(x);
  else if constexpr (ACT == kActSilu) {
    const float sg = 1.f / (1.f + __expf(-x));
    return sg * (1.f + x * (1.f - sg));
  } else if constexpr (ACT == kActTanh) {
    const float t = tanh_hw(x);
    return 1.f - t * t;
  } else return 1.f;
}

__device__ __forceinline__ float apply_act(int act, float x) {
  switch (act) {
    case kActRelu: return x > 0.f ? x : 0.f;
    case kActGelu: return gelu_erf_f(x);
    case kActGeluTanh: return gelu_tanh_f(x);
    case kActSilu: return x / (1.f + expf(-x));
    case kActTanh: return tanhf(x);
    default: return x;
  }
}

__device__ __forceinline__ float act_grad(int act, float x) {
  switch (act) {
    case kActRelu: return x > 0.f ? 1.f : 0.f;
    case kActGelu: return gelu_erf_grad_f(x);
    case kActGeluTanh: return gelu_tanh_grad_f(x);
    case kActSilu: {
      float s = 1.f / (1.f + expf(-x));
      return s * (1.f + x * (1.f - s));
    }
    case kActTanh: {
      float t = tanhf(x);
      return 1.f - t * t;
    }
    default: return 1.f;
  }
}

}  // namespace tgcm
