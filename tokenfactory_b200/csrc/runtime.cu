// Per-step runtime kernels around the hot path (engine/model_runner.py):
//  * req_to_token sync: the dirty segments of every request of a step in one launch
//    (ModelRunner._prepare_forward_batch, engine/model_runner.py:147-166);
//  * batched sampling: greedy argmax or an inverse-CDF draw from softmax(x / T) for every row in
//    one launch (ModelRunner._sample / _sample_one, engine/model_runner.py:574-581).
#include <math.h>

#include "common.cuh"
#include "launch.h"

namespace tf {
namespace rt {

// ---------------------------------------------------------------------------------------------
// req_to_token sync: one warp per segment, lane-strided int64 copies (rows are contiguous)
// ---------------------------------------------------------------------------------------------
__global__ void r2t_sync_kernel(tf_r2t_sync_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t s = warp; s < a.num_segments; s += nwarps) {
    const int64_t row = a.segments[4 * s], col = a.segments[4 * s + 1];
    const int64_t len = a.segments[4 * s + 2], src = a.segments[4 * s + 3];
    if (row < 0 || row >= a.r2t_rows || col < 0 || len < 0 || col + len > a.r2t_cols || src < 0 ||
        src + len > a.num_values) {
      if (lane == 0) record_err(a.err, TF_KERR_REQ_RANGE);
      continue;
    }
    int64_t* dst = a.req_to_token + row * a.r2t_stride + col;
    const int64_t* v = a.values + src;
    for (int64_t i = lane; i < len; i += 32) dst[i] = v[i];
  }
}

// ---------------------------------------------------------------------------------------------
// sampling: one CTA per row
// ---------------------------------------------------------------------------------------------
constexpr int kSampleThreads = 512;
constexpr int kWarps = kSampleThreads / 32;

// (value, index) order of torch.argmax: a NaN is the maximum, ties go to the smaller index
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  const bool vn = isnan(v), bn = isnan(bv);
  if (vn != bn) return vn;
  if (!vn && v != bv) return v > bv;
  return i < bi;
}

template <typename T, int E>
struct Row {  // E consecutive elements per thread per chunk, 16-byte loads when VEC
  const T* p;
  int n;
  bool vec;
  __device__ __forceinline__ void load(int base, float (&x)[E], int& cnt) const {
    cnt = n - base < E ? (n - base > 0 ? n - base : 0) : E;
    if (vec && cnt == E) {
      uint4 u[E * sizeof(T) / 16];
#pragma unroll
      for (int k = 0; k < (int)(E * sizeof(T) / 16); ++k)
        u[k] = __ldcs(reinterpret_cast<const uint4*>(p + base) + k);
      const T* e = reinterpret_cast<const T*>(u);
#pragma unroll
      for (int k = 0; k < E; ++k) x[k] = to_f(e[k]);
    } else {
#pragma unroll
      for (int k = 0; k < E; ++k) x[k] = k < cnt ? to_f(p[base + k]) : -INFINITY;
    }
  }
};

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < kWarps ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < kWarps ? red[lane] : -INFINITY;
  return warp_max(t);
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(tf_sample_args a, bool vec) {
  constexpr int E = 16 / sizeof(T) * (sizeof(T) == 2 ? 1 : 2);  // 8 elements per thread
  __shared__ float red[kWarps];
  __shared__ float wtot[kWarps];
  __shared__ int widx[kWarps];
  __shared__ float wval[kWarps];
  __shared__ int found;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const Row<T, E> row{reinterpret_cast<const T*>(a.logits) + (int64_t)b * a.logits_stride,
                      a.vocab_size, vec};
  const int chunk = kSampleThreads * E;
  const float temp = a.temperature[b];
  const bool greedy = a.uniform == nullptr || temp <= 1e-5f;

  // pass 1: argmax (greedy) or max
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int base = 0; base < a.vocab_size; base += chunk) {
    float x[E];
    int cnt;
    row.load(base + tid * E, x, cnt);
#pragma unroll
    for (int k = 0; k < E; ++k)
      if (k < cnt && better(x[k], base + tid * E + k, bv, bi)) { bv = x[k]; bi = base + tid * E + k; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { wval[w] = bv; widx[w] = bi; }
  __syncthreads();
  if (w == 0) {
    bv = lane < kWarps ? wval[lane] : -INFINITY;
    bi = lane < kWarps ? widx[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { wval[0] = bv; widx[0] = bi; }
  }
  __syncthreads();
  const float m = wval[0];
  if (greedy || isnan(m)) {
    if (tid == 0) a.out[b] = widx[0];
    return;
  }
  // pass 2: the normaliser
  const float it = 1.0f / temp;
  float s = 0.f;
  int last = -1;  // the largest index of nonzero weight (fallback when rounding leaves no crossing)
  for (int base = 0; base < a.vocab_size; base += chunk) {
    float x[E];
    int cnt;
    row.load(base + tid * E, x, cnt);
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const float e = k < cnt ? __expf((x[k] - m) * it) : 0.f;
      s += e;
      if (e > 0.f) last = base + tid * E + k;
    }
  }
  const float total = block_sum(s, red);
  last = __reduce_max_sync(0xffffffffu, last);
  __syncthreads();
  if (lane == 0) widx[w] = last;
  if (tid == 0) found = 0x7fffffff;
  __syncthreads();
  if (w == 0) {
    int l = lane < kWarps ? widx[lane] : -1;
    l = __reduce_max_sync(0xffffffffu, l);
    if (lane == 0) widx[0] = l;
  }
  const float target = a.uniform[b] * total;
  // pass 3: the first index whose running sum exceeds the target, chunk by chunk in index order
  float run = 0.f;
  for (int base = 0; base < a.vocab_size; base += chunk) {
    float x[E], e[E];
    int cnt;
    row.load(base + tid * E, x, cnt);
    float ts = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      e[k] = k < cnt ? __expf((x[k] - m) * it) : 0.f;
      ts += e[k];
    }
    // exclusive prefix of the thread sums across the CTA
    float incl = ts;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) wtot[w] = incl;
    __syncthreads();
    float wpre = 0.f, ctot = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) {
      const float t = wtot[k];
      wpre += k < w ? t : 0.f;
      ctot += t;
    }
    float acc = run + wpre + incl - ts;
    if (acc <= target && target < acc + ts) {
      int pick = base + tid * E + cnt - 1;
#pragma unroll
      for (int k = 0; k < E; ++k) {
        acc += e[k];
        if (k < cnt && acc > target) { pick = base + tid * E + k; break; }
      }
      atomicMin(&found, pick);
    }
    __syncthreads();
    if (found != 0x7fffffff) break;
    run += ctot;
  }
  if (tid == 0) a.out[b] = found != 0x7fffffff ? found : (widx[0] >= 0 ? widx[0] : 0);
}

}  // namespace rt

cudaError_t launch_req_to_token_sync(const tf_r2t_sync_args& a, cudaStream_t s) {
  if (a.num_segments == 0) return cudaSuccess;
  const int threads = 256;
  int64_t blocks = ((int64_t)a.num_segments * 32 + threads - 1) / threads;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  rt::r2t_sync_kernel<<<(int)blocks, threads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_sample_tokens(const tf_sample_args& a, cudaStream_t s) {
  if (a.batch_size == 0) return cudaSuccess;
  const int eb = a.dtype == TF_DTYPE_F32 ? 4 : 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(a.logits) | (uintptr_t)(a.logits_stride * eb)) & 15) == 0;
  if (a.dtype == TF_DTYPE_F32)
    rt::sample_kernel<float><<<a.batch_size, rt::kSampleThreads, 0, s>>>(a, vec);
  else if (a.dtype == TF_DTYPE_BF16)
    rt::sample_kernel<__nv_bfloat16><<<a.batch_size, rt::kSampleThreads, 0, s>>>(a, vec);
  else
    rt::sample_kernel<__half><<<a.batch_size, rt::kSampleThreads, 0, s>>>(a, vec);
  return cudaGetLastError();
}

}  // namespace tf
