// Shared device helpers for the tokenFactory B200 hot-path kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tfattn.h"

namespace tf {

// ---------------------------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Round a float to the precision of T and back (models a torch op whose result tensor is T).
template <typename T> __device__ __forceinline__ float round_to(float x) { return to_f(from_f<T>(x)); }

// Two floats rounded to a 16-bit T by one paired conversion (the same round-to-nearest-even as
// two from_f), packed with `a` in the low half; unpack_lo / unpack_hi read them back as floats.
// Conversions issue on a narrow pipe, so rows of 16-bit values are rounded and kept in pairs.
template <typename T> __device__ __forceinline__ uint32_t pack2_rn(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2_rn<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2_rn<__half>(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T> __device__ __forceinline__ float unpack_lo(uint32_t u);
template <typename T> __device__ __forceinline__ float unpack_hi(uint32_t u);
template <> __device__ __forceinline__ float unpack_lo<__nv_bfloat16>(uint32_t u) {
  return __uint_as_float(u << 16);
}
template <> __device__ __forceinline__ float unpack_hi<__nv_bfloat16>(uint32_t u) {
  return __uint_as_float(u & 0xffff0000u);
}
template <> __device__ __forceinline__ float unpack_lo<__half>(uint32_t u) {
  return __half2float(__ushort_as_half((unsigned short)(u & 0xffffu)));
}
template <> __device__ __forceinline__ float unpack_hi<__half>(uint32_t u) {
  return __half2float(__ushort_as_half((unsigned short)(u >> 16)));
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }

// torch.nn.functional.softplus (beta 1, threshold 20)
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

// out = attn * act(gate), both products rounded like bf16/f16 torch ops (full_attention.py:157-158)
template <typename T>
__device__ __forceinline__ float apply_gate(float attn_rounded, float gate, int mode) {
  if (mode == TF_GATE_NONE) return attn_rounded;
  float act = mode == TF_GATE_SILU ? silu_f(gate) : sigmoid_f(gate);
  return round_to<T>(attn_rounded * round_to<T>(act));
}

// ---------------------------------------------------------------------------------------------
// index handling shared by every kernel that reads the pools
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void record_err(int32_t* err, int32_t code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// req_to_token entry -> slot, mirroring the reference's clamp (batched path) or wrap (bsz==1 path);
// an entry outside the pool is recorded and read as slot 0 so the access stays in bounds.
__device__ __forceinline__ int64_t resolve_slot(int64_t s, int64_t num_slots, int slot_mode,
                                                int32_t* err) {
  if (s < 0) s = (slot_mode == TF_SLOT_WRAP) ? s + num_slots : 0;
  if (s < 0 || s >= num_slots) {
    record_err(err, TF_KERR_SLOT_RANGE);
    s = 0;
  }
  return s;
}

// ---------------------------------------------------------------------------------------------
// warp / block reductions
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------------------------
// bounded waits: every spin in these kernels ends after kSpinLimitNs and reports a timeout
// ---------------------------------------------------------------------------------------------
constexpr uint64_t kSpinLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after kSpinLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 255u) == 255u && global_ns() - t0 > kSpinLimitNs) return false;
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// 1-D bulk copy (TMA engine) global -> this CTA's shared memory, completing `bytes` on `bar`.
// dst, src and bytes must be multiples of 16; the source is this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// cp.async 16 B global -> shared, L1 bypass
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// 16-byte copy that reads `src_bytes` (0 or 16) bytes and zero-fills the rest
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
// arrive on `bar` once all prior cp.async of this thread have landed (counts as one arrival)
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace tf
