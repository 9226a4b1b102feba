// Block-FP8 linear of the reference (qwen3_8/fp8_triton.py: the wrapper :109-181 and the kernel
// :17-98, called by Qwen3_8FP8Linear._linear_op, qwen3_8/fp8_linear.py:181-201):
//  * tf_fp8_quantize: dynamic per-tensor activation scale and the e4m3 activations, bit-exact with
//    the wrapper's torch lines (amax in the activation dtype, the division by 448 in that dtype,
//    an IEEE fp32 division per element, clamp, round to nearest even);
//  * tf_fp8_block_gemm: out = (sum over 128-wide K blocks of (q . w^T)_block * w_scale[n/bh, k/bw])
//    * x_scale + bias on the 5th-generation tensor cores (tcgen05.mma kind::f8f6f4, e4m3 x e4m3 ->
//    fp32 in TMEM).  A 128 x 128 output tile meets one weight-scale block per K block (bh and bw
//    are multiples of 128), so each K block's product goes to its own TMEM accumulator (four in
//    rotation) and eight epilogue warps add it, times its scale, into fp32 registers while the
//    tensor core works on the next blocks.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace tf {
namespace fp8 {

// ---------------------------------------------------------------------------------------------
// activation quantization
// ---------------------------------------------------------------------------------------------
// x_scale = float(T(max(amax, 1e-12) / 448)): the wrapper's `amax.clamp(min=1e-12)` and `/ fp8_max`
// run on a tensor of the activation dtype (each rounded to it), then `.to(torch.float32)`
template <typename T>
__device__ __forceinline__ float act_scale(float amax) {
  const float c = round_to<T>(fmaxf(amax, 1e-12f));
  return round_to<T>(__fdiv_rn(c, 448.0f));
}

// two e4m3 values, round to nearest even (inputs already clamped to +-448); lo at the lower address
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// 16-byte vectors of a row: 8 elements of a 16-bit type, 4 of fp32
template <typename T> struct Vec { static constexpr int kN = 16 / sizeof(T); };

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[Vec<T>::kN]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int j = 0; j < Vec<T>::kN; ++j) v[j] = to_f(e[j]);
}

// A warp's unit of work: a row and a span of kSpan elements of it (lane-strided 16-byte vectors)
constexpr int kSpan = 1024;

// max |x| of this thread's share of the units warp0, warp0 + nwarps, ...
template <typename T>
__device__ __forceinline__ float thread_amax(const T* x, int64_t stride, int64_t M, int K,
                                             int64_t warp0, int64_t nwarps, int lane) {
  constexpr int V = Vec<T>::kN;
  const int spans = (K + kSpan - 1) / kSpan;
  float m = 0.f;
  for (int64_t u = warp0; u < M * spans; u += nwarps) {
    const int64_t r = u / spans;
    const int c1 = (int)(u - r * spans) * kSpan, c2 = c1 + kSpan < K ? c1 + kSpan : K;
    const T* row = x + r * stride;
    for (int c = c1 + lane * V; c < c2; c += 32 * V) {
      float v[V];
      load_vec(row + c, v);
#pragma unroll
      for (int j = 0; j < V; ++j) m = fmaxf(m, fabsf(v[j]));
    }
  }
  return warp_max(m);
}

template <typename T>
__device__ __forceinline__ void quantize_rows(const T* x, int64_t stride, int64_t M, int K, float s,
                                              uint8_t* q, int64_t warp0, int64_t nwarps, int lane) {
  constexpr int V = Vec<T>::kN;
  const int spans = (K + kSpan - 1) / kSpan;
  for (int64_t u = warp0; u < M * spans; u += nwarps) {
    const int64_t r = u / spans;
    const int c1 = (int)(u - r * spans) * kSpan, c2 = c1 + kSpan < K ? c1 + kSpan : K;
    const T* row = x + r * stride;
    uint8_t* qr = q + r * K;
    for (int c = c1 + lane * V; c < c2; c += 32 * V) {
      float v[V];
      load_vec(row + c, v);
      uint16_t pk[V / 2];
#pragma unroll
      for (int j = 0; j < V / 2; ++j) {
        const float a0 = fminf(fmaxf(__fdiv_rn(v[2 * j], s), -448.f), 448.f);
        const float a1 = fminf(fmaxf(__fdiv_rn(v[2 * j + 1], s), -448.f), 448.f);
        pk[j] = e4m3x2(a0, a1);
      }
      if constexpr (V == 8) {
        *reinterpret_cast<uint2*>(qr + c) = *reinterpret_cast<const uint2*>(pk);
      } else {
        *reinterpret_cast<uint32_t*>(qr + c) = *reinterpret_cast<const uint32_t*>(pk);
      }
    }
  }
}

// large inputs: amax over the grid (one atomic per warp; non-negative floats order as their bits)
template <typename T>
__global__ void amax_kernel(const T* x, int64_t stride, int64_t M, int K, unsigned int* amax_bits) {
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float m = thread_amax(x, stride, M, K, warp0, nwarps, threadIdx.x & 31);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

template <typename T>
__global__ void quantize_kernel(const T* x, int64_t stride, int64_t M, int K,
                                const unsigned int* amax_bits, uint8_t* q, float* x_scale) {
  const float s = act_scale<T>(__uint_as_float(*amax_bits));
  if (blockIdx.x == 0 && threadIdx.x == 0) *x_scale = s;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  quantize_rows(x, stride, M, K, s, q, warp0, nwarps, threadIdx.x & 31);
}

// small inputs (decode batches): one CTA computes the amax and quantizes, in one launch
template <typename T>
__global__ void __launch_bounds__(1024) quantize_small_kernel(const T* x, int64_t stride, int64_t M,
                                                              int K, uint8_t* q, float* x_scale) {
  __shared__ float red[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float m = thread_amax(x, stride, M, K, warp, nw, lane);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_max(t);
  const float s = act_scale<T>(t);
  if (threadIdx.x == 0) *x_scale = s;
  quantize_rows(x, stride, M, K, s, q, warp, nw, lane);
}

// ---------------------------------------------------------------------------------------------
// block-scaled GEMM
// ---------------------------------------------------------------------------------------------
constexpr int kBM = 128, kBN = 128, kBK = 128;  // a K block is one 128-byte SW128 row per operand row
constexpr int kStages = 4;
constexpr int kTile = kBM * kBK;                // 16 KB per operand per stage
constexpr int kStageBytes = 2 * kTile;
constexpr int kThreads = 320;                   // warps 0-7 epilogue, 8 MMA, 9 TMA loads
constexpr int kMmaWarp = 8, kLoadWarp = 9;
constexpr int kAcc = 4;                         // TMEM accumulators of 128 columns (all 512)
constexpr int kSmem = kStages * kStageBytes + 256 + 1024;

struct Bars {
  uint64_t full[kStages], empty[kStages], pfull[kAcc], pfree[kAcc], fin;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(Bars) <= 256, "barriers overflow their shared-memory slot");

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

// 2-D tiled TMA load of one 128 x 128-byte box (SWIZZLE_128B) into this CTA's shared memory;
// the source is this GPU's own memory and the x coordinate (bytes) is a multiple of 128
__device__ __forceinline__ void tma_load_box(uint32_t dst, const CUtensorMap* map, int x, int y,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// the epilogue warps wait most of the time: back off so that their polling leaves the issue
// slots to the MMA and TMA threads on the same SM sub-partitions
__device__ __forceinline__ bool wait_b_backoff(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(64);
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 15u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kSpinLimitNs) { *abort = 1; return false; }
    }
  }
}

template <typename TO>
__global__ void __launch_bounds__(kThreads, 1) block_gemm_kernel(tf_fp8_gemm_args a,
                                                                 const __grid_constant__ CUtensorMap map_q,
                                                                 const __grid_constant__ CUtensorMap map_w) {
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
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(&bars->pfull[b], 1);
      mbar_init(&bars->pfree[b], 8);
    }
    mbar_init(&bars->fin, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tc::tmem_alloc(&bars->tmem, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp == kLoadWarp) {
    // ============ loads: two TMA boxes (q rows, w rows; zero fill past M, N and K) per stage ============
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !wait_b(&bars->empty[s], ((kb / kStages) - 1) & 1, abort)) break;
        const uint32_t st = base + s * kStageBytes;
        mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
        tma_load_box(st, &map_q, kb * kBK, (int)m0, &bars->full[s]);
        tma_load_box(st + kTile, &map_w, kb * kBK, n0, &bars->full[s]);
        issued = kb + 1;
      }
      // after an abort, boxes still in flight land (bounded wait) before the CTA ends
      for (int kb = issued - kStages > 0 ? issued - kStages : 0; kb < issued; ++kb)
        mbar_wait(&bars->full[kb % kStages], (kb / kStages) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ============ MMA issue (one thread): one K block into one of four TMEM accumulators ============
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4)                       // D: f32
                                 | (0u << 7) | (0u << 10)         // A, B: e4m3
                                 | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages, b = kb % kAcc;
        if (!wait_b(&bars->full[s], (kb / kStages) & 1, abort)) break;
        if (kb >= kAcc && !wait_b(&bars->pfree[b], ((kb / kAcc) - 1) & 1, abort)) break;
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
      // every MMA issued has completed before TMEM is released, also after an abort (bounded)
      tc::commit(&bars->fin);
      mbar_wait(&bars->fin, 0);
    }
    __syncwarp();
  } else {
    // ============ epilogue: acc += w_scale * partial per K block, then out = acc * x_scale + bias ============
    // warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and columns 64 (w / 4) .. +63
    const int q = warp & 3, h = warp >> 2;
    const int row = 32 * q + lane;
    const uint32_t lb = tmem + ((uint32_t)(32 * q) << 16) + 64 * h;
    const float* wsrow = a.w_scale ? a.w_scale + (int64_t)(n0 / a.block_h) * a.ws_stride_n : nullptr;
    auto scale_of = [&](int kb) -> float {
      return wsrow ? __ldg(wsrow + (int64_t)(kb * kBK / a.block_w) * a.ws_stride_k) : 1.f;
    };
    float acc[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    bool ok = true;
    float sc_next = scale_of(0);
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int b = kb % kAcc;
      const float sc = sc_next;
      if (kb + 1 < nkb) sc_next = scale_of(kb + 1);  // in flight while this block's MMAs finish
      ok = wait_b_backoff(&bars->pfull[b], (kb / kAcc) & 1, abort);
      if (!ok) break;
      tc::fence_after_sync();
      float p[64];
      tc::ld32(lb + b * 128, *reinterpret_cast<float(*)[32]>(&p[0]));
      tc::ld32(lb + b * 128 + 32, *reinterpret_cast<float(*)[32]>(&p[32]));
      tc::wait_ld();
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = fmaf(p[j], sc, acc[j]);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->pfree[b]);
    }
    if (ok && m0 + row < a.M) {
      const float xs = *a.x_scale;
      const int c0 = 64 * h;
      TO* out = reinterpret_cast<TO*>(a.out) + (m0 + row) * a.out_stride + n0 + c0;
      const int ncol = a.N - n0 - c0 < 64 ? a.N - n0 - c0 : 64;
      const bool vec = ncol == 64 && ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && sizeof(TO) == 2;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int n = c8 * 8 + e;
          float bias = 0.f;
          if (a.bias && n < ncol) {
            const int64_t bn = n0 + c0 + n;
            bias = a.bias_dtype == TF_DTYPE_F32 ? reinterpret_cast<const float*>(a.bias)[bn]
                 : a.bias_dtype == TF_DTYPE_BF16 ? to_f(reinterpret_cast<const __nv_bfloat16*>(a.bias)[bn])
                                                 : to_f(reinterpret_cast<const __half*>(a.bias)[bn]);
          }
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
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------------------
// Prefill-sized M: 128 x 256 tiles, one persistent CTA per SM.  A K block of a 256-column tile
// moves 48 KB (16 KB of q, 32 KB of w) for twice the products of a 128 x 128 tile's 32 KB, a
// quarter less L2 -> SM traffic per product, which is what bounds the 128 x 128 kernel.  Each CTA
// walks the tiles blockIdx.x, blockIdx.x + gridDim.x, ... (m fastest: the CTAs resident at once
// share a few 256-row weight blocks and re-read the activations, which stay in L2, instead of
// streaming the whole weight matrix from DRAM once per two row blocks), with one running count of
// K blocks for the stage ring and the accumulator pair, so the next tile's loads and first
// products overlap the current tile's output writes.  TMEM holds two 256-column accumulators;
// epilogue warp w reads lanes 32 (w % 4) .. +31 and the 128 columns 128 (w / 4) .. +127, the span
// of one weight-scale row block (block_h is a multiple of 128).
// ---------------------------------------------------------------------------------------------
constexpr int kBNW = 256;
constexpr int kStagesW = 4;
constexpr int kTileW = kBNW * kBK;              // 32 KB of w rows per stage
constexpr int kStageBytesW = kTile + kTileW;    // 48 KB
constexpr int kAccW = 2;                        // TMEM accumulators of 256 columns (all 512)
constexpr int kSmemW = kStagesW * kStageBytesW + 256 + 1024;
static_assert(kSmemW <= 232448, "shared memory per CTA");

struct BarsW {
  uint64_t full[kStagesW], empty[kStagesW], pfull[kAccW], pfree[kAccW], fin;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(BarsW) <= 256, "barriers overflow their shared-memory slot");

template <typename TO>
__global__ void __launch_bounds__(kThreads, 1) block_gemm_wide_kernel(tf_fp8_gemm_args a,
                                                                      const __grid_constant__ CUtensorMap map_q,
                                                                      const __grid_constant__ CUtensorMap map_w,
                                                                      int tiles_m, int tiles) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  unsigned char* sb = smem_raw + (base - raw);
  BarsW* bars = reinterpret_cast<BarsW*>(sb + kStagesW * kStageBytesW);
  volatile int* abort = &bars->abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = (a.K + kBK - 1) / kBK;

  if (tid == 0) {
    for (int s = 0; s < kStagesW; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < kAccW; ++b) {
      mbar_init(&bars->pfull[b], 1);
      mbar_init(&bars->pfree[b], 8);
    }
    mbar_init(&bars->fin, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tc::tmem_alloc(&bars->tmem, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp == kLoadWarp) {
    // ============ loads: a q box and a 256-row w box per stage, over all of this CTA's tiles ============
    if (lane == 0) {
      uint32_t g = 0;  // K blocks issued so far
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t % tiles_m) * kBM, n0 = (t / tiles_m) * kBNW;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const uint32_t s = g % kStagesW;
          if (g >= kStagesW && !wait_b(&bars->empty[s], ((g / kStagesW) - 1) & 1, abort)) {
            ok = false;
            break;
          }
          const uint32_t st = base + s * kStageBytesW;
          mbar_arrive_expect_tx(&bars->full[s], kStageBytesW);
          tma_load_box(st, &map_q, kb * kBK, m0, &bars->full[s]);
          tma_load_box(st + kTile, &map_w, kb * kBK, n0, &bars->full[s]);
        }
      }
      // after an abort, boxes still in flight land (bounded wait) before the CTA ends
      for (uint32_t j = g > (uint32_t)kStagesW ? g - kStagesW : 0; j < g; ++j)
        mbar_wait(&bars->full[j % kStagesW], (j / kStagesW) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ============ MMA issue (one thread): K block g into accumulator g % 2 ============
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4)                       // D: f32
                                 | (0u << 7) | (0u << 10)         // A, B: e4m3
                                 | ((uint32_t)(kBNW >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const uint32_t s = g % kStagesW, b = g % kAccW;
          if (!wait_b(&bars->full[s], (g / kStagesW) & 1, abort) ||
              (g >= kAccW && !wait_b(&bars->pfree[b], ((g / kAccW) - 1) & 1, abort))) {
            ok = false;
            break;
          }
          tc::fence_proxy_async_smem();
          tc::fence_after_sync();
          const uint32_t st = base + s * kStageBytesW;
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {  // K = 32 e4m3 values = 32 bytes per MMA
            const uint64_t da = tc::sw128_desc(st + kk * 32, 16, 1024);
            const uint64_t db = tc::sw128_desc(st + kTile + kk * 32, 16, 1024);
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem + b * kBNW),
                "l"(da), "l"(db), "r"(idesc), "r"(kk > 0 ? 1u : 0u)
                : "memory");
          }
          tc::commit(&bars->empty[s]);
          tc::commit(&bars->pfull[b]);
        }
      }
      // every MMA issued has completed before TMEM is released, also after an abort (bounded)
      tc::commit(&bars->fin);
      mbar_wait(&bars->fin, 0);
    }
    __syncwarp();
  } else {
    // ============ epilogue: acc += w_scale * partial per K block, then out = acc * x_scale + bias ============
    const int q = warp & 3, h = warp >> 2;
    const int row = 32 * q + lane;
    const uint32_t lb = tmem + ((uint32_t)(32 * q) << 16) + 128 * h;
    uint32_t g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const int n0 = (t / tiles_m) * kBNW + 128 * h;  // this warp's first column
      const int64_t m0 = (int64_t)(t % tiles_m) * kBM;
      // a half that starts past N has no output columns and reads no weight scale
      const float* wsrow = a.w_scale && n0 < a.N ? a.w_scale + (int64_t)(n0 / a.block_h) * a.ws_stride_n
                                                 : nullptr;
      auto scale_of = [&](int kb) -> float {
        return wsrow ? __ldg(wsrow + (int64_t)(kb * kBK / a.block_w) * a.ws_stride_k) : 1.f;
      };
      float acc[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.f;
      float sc_next = scale_of(0);
      for (int kb = 0; kb < nkb; ++kb, ++g) {
        const uint32_t b = g % kAccW;
        const float sc = sc_next;
        if (kb + 1 < nkb) sc_next = scale_of(kb + 1);  // in flight while this block's MMAs finish
        if (!wait_b_backoff(&bars->pfull[b], (g / kAccW) & 1, abort)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float p[32];
          tc::ld32(lb + b * kBNW + 32 * c, p);
          tc::wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[32 * c + j] = fmaf(p[j], sc, acc[32 * c + j]);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->pfree[b]);
      }
      if (!ok || m0 + row >= a.M || n0 >= a.N) continue;
      const float xs = *a.x_scale;
      TO* out = reinterpret_cast<TO*>(a.out) + (m0 + row) * a.out_stride + n0;
      const int ncol = a.N - n0 < 128 ? a.N - n0 : 128;
      const bool vec = ncol == 128 && ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && sizeof(TO) == 2;
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int n = c8 * 8 + e;
          float bias = 0.f;
          if (a.bias && n < ncol) {
            const int64_t bn = n0 + n;
            bias = a.bias_dtype == TF_DTYPE_F32 ? reinterpret_cast<const float*>(a.bias)[bn]
                 : a.bias_dtype == TF_DTYPE_BF16 ? to_f(reinterpret_cast<const __nv_bfloat16*>(a.bias)[bn])
                                                 : to_f(reinterpret_cast<const __half*>(a.bias)[bn]);
          }
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
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, 512);
}

}  // namespace fp8

size_t fp8_quantize_workspace() { return 256; }

template <typename T>
cudaError_t quantize_t(const tf_fp8_quant_args& a, cudaStream_t s) {
  const T* x = static_cast<const T*>(a.x);
  const int64_t n = a.M * (int64_t)a.K;
  if (n <= (int64_t)1 << 15) {  // up to 32K elements: one CTA, one launch
    fp8::quantize_small_kernel<T><<<1, 1024, 0, s>>>(x, a.x_stride, a.M, a.K, a.q, a.x_scale);
    return cudaGetLastError();
  }
  unsigned int* amax = static_cast<unsigned int*>(a.workspace);
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess) return e;
  const int64_t units = a.M * ((a.K + fp8::kSpan - 1) / fp8::kSpan);
  const int64_t warps = units < (int64_t)device_sm_count() * 64 ? units : (int64_t)device_sm_count() * 64;
  const int grid = (int)((warps * 32 + 255) / 256);
  fp8::amax_kernel<T><<<grid, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax);
  fp8::quantize_kernel<T><<<grid, 256, 0, s>>>(x, a.x_stride, a.M, a.K, amax, a.q, a.x_scale);
  return cudaGetLastError();
}

cudaError_t launch_fp8_quantize(const tf_fp8_quant_args& a, cudaStream_t s) {
  if (a.M == 0 || a.K == 0) return cudaSuccess;
  switch (a.dtype) {
    case TF_DTYPE_BF16: return quantize_t<__nv_bfloat16>(a, s);
    case TF_DTYPE_F16: return quantize_t<__half>(a, s);
    default: return quantize_t<float>(a, s);
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [rows, cols] bytes with a row stride, read in boxes of 128 bytes x box_rows rows, SWIZZLE_128B,
// zero fill outside
bool box_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t stride,
             uint32_t box_rows = 128) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {(cuuint32_t)fp8::kBK, box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

template <typename TO>
cudaError_t gemm_t(const tf_fp8_gemm_args& a, cudaStream_t s) {
  CUtensorMap mq, mw;
  if (!box_map(&mq, a.q, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.q_stride))
    return cudaErrorNotSupported;
  // 128 x 256 tiles once they fill every SM at least once; smaller problems (decode batches) keep
  // the 128 x 128 tiles, which give twice as many CTAs to stream the weights
  const int sms = device_sm_count();
  const int64_t tiles_m = (a.M + fp8::kBM - 1) / fp8::kBM;
  const int64_t tiles_nw = (a.N + fp8::kBNW - 1) / fp8::kBNW;
  if (tiles_m * tiles_nw >= sms && tiles_m * tiles_nw <= INT32_MAX) {
    if (!box_map(&mw, a.w, (uint64_t)a.N, (uint64_t)a.K, (uint64_t)a.w_stride, fp8::kBNW))
      return cudaErrorNotSupported;
    cudaError_t e = cudaFuncSetAttribute(fp8::block_gemm_wide_kernel<TO>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, fp8::kSmemW);
    if (e != cudaSuccess) return e;
    const int tiles = (int)(tiles_m * tiles_nw);
    fp8::block_gemm_wide_kernel<TO><<<tiles < sms ? tiles : sms, fp8::kThreads, fp8::kSmemW, s>>>(
        a, mq, mw, (int)tiles_m, tiles);
    return cudaGetLastError();
  }
  if (!box_map(&mw, a.w, (uint64_t)a.N, (uint64_t)a.K, (uint64_t)a.w_stride))
    return cudaErrorNotSupported;
  dim3 grid((a.N + fp8::kBN - 1) / fp8::kBN, (unsigned)tiles_m);
  cudaError_t e = cudaFuncSetAttribute(fp8::block_gemm_kernel<TO>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, fp8::kSmem);
  if (e != cudaSuccess) return e;
  fp8::block_gemm_kernel<TO><<<grid, fp8::kThreads, fp8::kSmem, s>>>(a, mq, mw);
  return cudaGetLastError();
}

cudaError_t launch_fp8_block_gemm(const tf_fp8_gemm_args& a, cudaStream_t s) {
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  switch (a.out_dtype) {
    case TF_DTYPE_BF16: return gemm_t<__nv_bfloat16>(a, s);
    case TF_DTYPE_F16: return gemm_t<__half>(a, s);
    default: return gemm_t<float>(a, s);
  }
}

}  // namespace tf
