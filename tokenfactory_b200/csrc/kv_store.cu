// a1. KV-pool store: k_buffer[out_cache_loc[t]] = k[t] (and v), the pool write of
// qwen3_8/full_attention.py:147-149.  One warp per (token, kv head) row; 16-byte vector copies when
// row length and strides allow, element copies otherwise.  Bit-exact.
#include "common.cuh"
#include "launch.h"

namespace tf {

template <int VEC_BYTES>
__global__ void kv_store_kernel(tf_kv_store_args a, int elem_bytes) {
  const int64_t rows = a.num_tokens * (int64_t)a.num_kv_heads;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int row_bytes = a.head_dim * elem_bytes;
  const int nvec = row_bytes / VEC_BYTES;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const int64_t t = r / a.num_kv_heads;
    const int h = (int)(r - t * a.num_kv_heads);
    int64_t loc = a.out_cache_loc[t];
    if (loc < 0) loc += a.num_slots;  // torch index semantics
    if (loc < 0 || loc >= a.num_slots) {
      if (lane == 0) record_err(a.err, TF_KERR_SLOT_RANGE);
      continue;
    }
    const char* ks = (const char*)a.k + (t * a.k_stride_tok + h * a.k_stride_head) * elem_bytes;
    const char* vs = (const char*)a.v + (t * a.v_stride_tok + h * a.v_stride_head) * elem_bytes;
    const int64_t doff = (loc * a.buf_stride_slot + h * a.buf_stride_head) * elem_bytes;
    char* kd = (char*)a.k_buffer + doff;
    char* vd = (char*)a.v_buffer + doff;
    if (VEC_BYTES == 16) {
      for (int i = lane; i < nvec; i += 32) {
        reinterpret_cast<uint4*>(kd)[i] = __ldg(reinterpret_cast<const uint4*>(ks) + i);
        reinterpret_cast<uint4*>(vd)[i] = __ldg(reinterpret_cast<const uint4*>(vs) + i);
      }
    } else {
      for (int i = lane; i < row_bytes; i += 32) {
        kd[i] = ks[i];
        vd[i] = vs[i];
      }
    }
  }
}

cudaError_t launch_kv_store(const tf_kv_store_args& a, cudaStream_t s) {
  const int eb = a.dtype == TF_DTYPE_F32 ? 4 : 2;
  const int64_t rows = a.num_tokens * (int64_t)a.num_kv_heads;
  if (rows == 0) return cudaSuccess;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = ((int64_t)a.head_dim * eb) % 16 == 0 && al16(a.k) && al16(a.v) &&
                   al16(a.k_buffer) && al16(a.v_buffer) &&
                   (a.k_stride_tok * eb) % 16 == 0 && (a.k_stride_head * eb) % 16 == 0 &&
                   (a.v_stride_tok * eb) % 16 == 0 && (a.v_stride_head * eb) % 16 == 0 &&
                   (a.buf_stride_slot * eb) % 16 == 0 && (a.buf_stride_head * eb) % 16 == 0;
  const int threads = 256;
  int64_t blocks = (rows * 32 + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (vec)
    kv_store_kernel<16><<<(int)blocks, threads, 0, s>>>(a, eb);
  else
    kv_store_kernel<1><<<(int)blocks, threads, 0, s>>>(a, eb);
  return cudaGetLastError();
}

}  // namespace tf
