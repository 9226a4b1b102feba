// Block-FP8 linear of the reference (qwen3_8/fp8_triton.py: the wrapper :109-181 and the kernel
// :17-98, called by Qwen3_8FP8Linear._linear_op, qwen3_8/fp8_linear.py:181-201):
//  * tf_fp8_quantize: dynamic per-tensor activation scale and the e4m3 activations, bit-exact with
//    the wrapper's torch lines (amax in the activation dtype, the division by 448 in that dtype,
//    an IEEE fp32 division per element, clamp, round to nearest even);
//  * tf_fp8_block_gemm: out = (sum over 128-wide K blocks of (q . w^T)_block * w_scale[n/bh, k/bw])
//    * x_scale + bias on the 5th-generation tensor cores (tcgen05.mma kind::f8f6f4, e4m3 x e4m3 ->
//    fp32 in TMEM).  A 128 x 128 output tile meets one weight-scale block per K block (bh and bw
//    are multiples of 128), so each K block's product goes to its own TMEM accumulator (two,
//    alternating) and the epilogue warps add it, times its scale, into fp32 registers while the
//    tensor core works on the next block.
#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace tf {
namespace fp8 {

// ---------------------------------------------------------------------------------------------
// activation quantization
// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void amax_kernel(const T* x, int64_t stride, int64_t M, int K, unsigned int* amax_bits) {
  float m = 0.f;
  const int64_t n = M * (int64_t)K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K, c = i - r * K;
    m = fmaxf(m, fabsf(to_f(x[r * stride + c])));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));  // m >= 0: bit order = value order
}

// x_scale = float(T(max(amax, 1e-12) / 448)): the wrapper's `amax.clamp(min=1e-12)` and `/ fp8_max`
// run on a tensor of the activation dtype (each rounded to it), then `.to(torch.float32)`
template <typename T>
__device__ __forceinline__ float act_scale(float amax) {
  const float c = round_to<T>(fmaxf(amax, 1e-12f));
  return round_to<T>(__fdiv_rn(c, 448.0f));
}

__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T>
__global__ void quantize_kernel(const T* x, int64_t stride, int64_t M, int K,
                                const unsigned int* amax_bits, uint8_t* q, float* x_scale) {
  const float s = act_scale<T>(__uint_as_float(*amax_bits));
  if (blockIdx.x == 0 && threadIdx.x == 0) *x_scale = s;
  const int64_t pairs = M * (int64_t)(K / 2);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < pairs;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (K / 2), c = 2 * (i - r * (K / 2));
    const float a = fminf(fmaxf(__fdiv_rn(to_f(x[r * stride + c]), s), -448.f), 448.f);
    const float b = fminf(fmaxf(__fdiv_rn(to_f(x[r * stride + c + 1]), s), -448.f), 448.f);
    *reinterpret_cast<uint16_t*>(q + r * K + c) = e4m3x2(a, b);
  }
}

// ---------------------------------------------------------------------------------------------
// block-scaled GEMM
// ---------------------------------------------------------------------------------------------
constexpr int kBM = 128, kBN = 128, kBK = 128;  // a K block is one 128-byte SW128 row per operand row
constexpr int kStages = 4;
constexpr int kTile = kBM * kBK;                // 16 KB per operand per stage
constexpr int kStageBytes = 2 * kTile;
constexpr int kThreads = 256;                   // warps 0-3 epilogue, 4 MMA, 5-7 loads
constexpr int kLoaders = 96;
constexpr int kChunks = 2 * kBM * kBK / 16;     // 16-byte pieces per stage (A and B)
constexpr int kSmem = kStages * kStageBytes + 256 + 1024;

struct Bars {
  uint64_t full[kStages], empty[kStages], pfull[2], pfree[2];
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ bool wait_b(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kSpinLimitNs) { *abort = 1; return false; }
    }
  }
}

template <typename TO>
__global__ void __launch_bounds__(kThreads, 1) block_gemm_kernel(tf_fp8_gemm_args a) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* sb = smem_raw + (base - raw);
  Bars* bars = reinterpret_cast<Bars*>(sb + kStages * kStageBytes);
  volatile int* abort = &bars->abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.y * kBM;
  const int n0 = blockIdx.x * kBN;
  const int nkb = (a.K + kBK - 1) / kBK;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], kLoaders);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->pfull[b], 1);
      mbar_init(&bars->pfree[b], 4);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 4) tc::tmem_alloc(&bars->tmem, 256);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp >= 5) {
    // ============ loads: 16-byte cp.async into the SW128 K-major layout ============
    const int pt = tid - 160;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages && !wait_b(&bars->empty[s], ((kb / kStages) - 1) & 1, abort)) break;
      const uint32_t st = base + s * kStageBytes;
#pragma unroll 4
      for (int i = 0; i < (kChunks + kLoaders - 1) / kLoaders; ++i) {
        const int qid = pt + kLoaders * i;
        if (qid >= kChunks) break;
        const int op = qid >> 10, r = (qid >> 3) & 127, c = qid & 7;
        const int kbyte = kb * kBK + c * 16;
        const uint32_t dst = st + op * kTile + r * 128 + ((uint32_t)(c ^ (r & 7)) << 4);
        const bool live_k = kbyte < a.K;  // K is a multiple of 16: a chunk is all in or all out
        if (op == 0) {
          const bool live = live_k && m0 + r < a.M;
          const uint8_t* src = a.q + (live ? (m0 + r) * a.q_stride + kbyte : 0);
          cp_async16_zfill(dst, src, live ? 16u : 0u);
        } else {
          const bool live = live_k && n0 + r < a.N;
          const uint8_t* src = a.w + (live ? (int64_t)(n0 + r) * a.w_stride + kbyte : 0);
          cp_async16_zfill(dst, src, live ? 16u : 0u);
        }
      }
      cp_async_arrive_noinc(&bars->full[s]);
    }
    cp_async_wait_all();
  } else if (warp == 4) {
    // ============ MMA issue (one thread): one K block into one of two TMEM accumulators ============
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4)                       // D: f32
                                 | (0u << 7) | (0u << 10)         // A, B: e4m3
                                 | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages, b = kb & 1;
        if (!wait_b(&bars->full[s], (kb / kStages) & 1, abort)) break;
        if (kb >= 2 && !wait_b(&bars->pfree[b], ((kb >> 1) - 1) & 1, abort)) break;
        tc::fence_proxy_async_smem();
        tc::fence_after_sync();
        const uint32_t st = base + s * kStageBytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 32; ++kk) {  // K = 32 e4m3 values = 32 bytes per MMA
          const uint64_t da = tc::sw128_desc(st + kk * 32, 16, 1024);
          const uint64_t db = tc::sw128_desc(st + kTile + kk * 32, 16, 1024);
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem + b * 128),
              "l"(da), "l"(db), "r"(idesc), "r"(kk > 0 ? 1u : 0u)
              : "memory");
        }
        tc::commit(&bars->empty[s]);
        tc::commit(&bars->pfull[b]);
      }
    }
    __syncwarp();
  } else {
    // ============ epilogue: acc += w_scale * partial per K block, then out = acc * x_scale + bias ============
    const int row = 32 * warp + lane;  // TMEM lane = output row of the tile
    const uint32_t lb = tmem + ((uint32_t)(32 * warp) << 16);
    float acc[kBN];
#pragma unroll
    for (int j = 0; j < kBN; ++j) acc[j] = 0.f;
    bool ok = true;
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int b = kb & 1;
      ok = wait_b(&bars->pfull[b], (kb >> 1) & 1, abort);
      if (!ok) break;
      tc::fence_after_sync();
      float sc = 1.f;
      if (a.w_scale)
        sc = a.w_scale[(int64_t)(n0 / a.block_h) * a.ws_stride_n + (int64_t)(kb * kBK / a.block_w) * a.ws_stride_k];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        float p[32];
        tc::ld32(lb + b * 128 + 32 * c, p);
        tc::wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[32 * c + j] = fmaf(p[j], sc, acc[32 * c + j]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->pfree[b]);
    }
    if (ok && m0 + row < a.M) {
      const float xs = *a.x_scale;
      TO* out = reinterpret_cast<TO*>(a.out) + (m0 + row) * a.out_stride + n0;
      const int ncol = a.N - n0 < kBN ? a.N - n0 : kBN;
      const bool vec = ncol == kBN && ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && sizeof(TO) == 2;
#pragma unroll
      for (int c8 = 0; c8 < kBN / 8; ++c8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int n = c8 * 8 + e;
          float bias = 0.f;
          if (a.bias && n < ncol)
            bias = a.bias_dtype == TF_DTYPE_F32 ? reinterpret_cast<const float*>(a.bias)[n0 + n]
                 : a.bias_dtype == TF_DTYPE_BF16 ? to_f(reinterpret_cast<const __nv_bfloat16*>(a.bias)[n0 + n])
                                                 : to_f(reinterpret_cast<const __half*>(a.bias)[n0 + n]);
          v[e] = fmaf(acc[n], xs, bias);
        }
        if (vec) {
          TO pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) pk[e] = from_f<TO>(v[e]);
          *reinterpret_cast<uint4*>(out + c8 * 8) = *reinterpret_cast<const uint4*>(pk);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c8 * 8 + e < ncol) out[c8 * 8 + e] = from_f<TO>(v[e]);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && *abort && a.err) record_err(a.err, TF_KERR_TIMEOUT);
  tc::fence_after_sync();
  if (warp == 4) tc::tmem_dealloc(tmem, 256);
}

}  // namespace fp8

size_t fp8_quantize_workspace() { return 256; }

cudaError_t launch_fp8_quantize(const tf_fp8_quant_args& a, cudaStream_t s) {
  if (a.M == 0 || a.K == 0) return cudaSuccess;
  unsigned int* amax = static_cast<unsigned int*>(a.workspace);
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess) return e;
  const int64_t n = a.M * (int64_t)a.K;
  const int cap = device_sm_count() * 8;
  const int g1 = (int)((n + 255) / 256 < cap ? (n + 255) / 256 : cap);
  const int g2 = (int)((n / 2 + 255) / 256 < cap ? (n / 2 + 255) / 256 : cap);
  switch (a.dtype) {
    case TF_DTYPE_BF16: {
      auto x = static_cast<const __nv_bfloat16*>(a.x);
      fp8::amax_kernel<<<g1, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax);
      fp8::quantize_kernel<<<g2, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax, a.q, a.x_scale);
      break;
    }
    case TF_DTYPE_F16: {
      auto x = static_cast<const __half*>(a.x);
      fp8::amax_kernel<<<g1, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax);
      fp8::quantize_kernel<<<g2, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax, a.q, a.x_scale);
      break;
    }
    default: {
      auto x = static_cast<const float*>(a.x);
      fp8::amax_kernel<<<g1, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax);
      fp8::quantize_kernel<<<g2, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax, a.q, a.x_scale);
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_fp8_block_gemm(const tf_fp8_gemm_args& a, cudaStream_t s) {
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  dim3 grid((a.N + fp8::kBN - 1) / fp8::kBN, (unsigned)((a.M + fp8::kBM - 1) / fp8::kBM));
  cudaError_t e;
  switch (a.out_dtype) {
    case TF_DTYPE_BF16:
      e = cudaFuncSetAttribute(fp8::block_gemm_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, fp8::kSmem);
      if (e != cudaSuccess) return e;
      fp8::block_gemm_kernel<__nv_bfloat16><<<grid, fp8::kThreads, fp8::kSmem, s>>>(a);
      break;
    case TF_DTYPE_F16:
      e = cudaFuncSetAttribute(fp8::block_gemm_kernel<__half>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, fp8::kSmem);
      if (e != cudaSuccess) return e;
      fp8::block_gemm_kernel<__half><<<grid, fp8::kThreads, fp8::kSmem, s>>>(a);
      break;
    default:
      e = cudaFuncSetAttribute(fp8::block_gemm_kernel<float>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, fp8::kSmem);
      if (e != cudaSuccess) return e;
      fp8::block_gemm_kernel<float><<<grid, fp8::kThreads, fp8::kSmem, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace tf
