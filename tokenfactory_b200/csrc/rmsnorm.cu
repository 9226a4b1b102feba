// a9 standalone: out = w * x/rms_head(x) * silu(z) in fp32, rounded to the activation dtype
// (qwen3_8/rms_norm_gated.py:26-40).  One warp per (token, head).  The GDN kernels fuse the same
// epilogue; this entry point serves callers that hold x already.
#include "common.cuh"
#include "launch.h"

namespace tf {

template <typename T>
__global__ void __launch_bounds__(256) gated_rmsnorm_kernel(tf_gated_rmsnorm_args a) {
  const int64_t rows = (int64_t)a.num_tokens * a.num_heads;
  const int lane = threadIdx.x & 31;
  const int64_t wid = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (wid >= rows) return;
  const int64_t t = wid / a.num_heads;
  const int h = (int)(wid - t * a.num_heads);
  const int hd = a.head_dim;
  const T* x = reinterpret_cast<const T*>(a.x) + t * a.x_stride_tok + (int64_t)h * hd;
  const T* z = reinterpret_cast<const T*>(a.z) + t * a.z_stride_tok + (int64_t)h * hd;
  const T* w = reinterpret_cast<const T*>(a.weight) + (a.weight_len == hd ? 0 : (int64_t)h * hd);
  T* out = reinterpret_cast<T*>(a.out) + t * a.out_stride_tok + (int64_t)h * hd;
  float ss = 0.f;
  for (int j = lane; j < hd; j += 32) {
    const float v = to_f(x[j]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)hd + a.eps);
  for (int j = lane; j < hd; j += 32)
    out[j] = from_f<T>(to_f(w[j]) * (to_f(x[j]) * rs) * silu_f(to_f(z[j])));
}

cudaError_t launch_gated_rmsnorm(const tf_gated_rmsnorm_args& a, cudaStream_t s) {
  const int64_t rows = (int64_t)a.num_tokens * a.num_heads;
  if (rows == 0) return cudaSuccess;
  const int64_t blocks = (rows * 32 + 255) / 256;
  switch (a.dtype) {
    case TF_DTYPE_F32: gated_rmsnorm_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(a); break;
    case TF_DTYPE_BF16: gated_rmsnorm_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(a); break;
    default: gated_rmsnorm_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace tf
