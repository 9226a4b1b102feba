// a2/a3 generic path: paged GQA attention on CUDA cores for any dtype (fp32 / bf16 / fp16) and any
// head_dim <= 256.  Serves the fp32 configurations (the reference runs fp32 on CPU), head dims the
// tensor-core kernels are not built for, and extend batches.  One CTA per (query token, kv head)
// computes the G = Hq/Hkv query heads that share the kv head, so every K/V row is read once per
// group.  Semantics follow qwen3_8/full_attention.py:163-283 (see tfattn.h).
#include "common.cuh"
#include "launch.h"

namespace tf {

namespace {
constexpr int kThreads = 128;
constexpr int kBK = 32;  // keys per block

// Request b of token t and the first token of b, found by one warp from extend_lens.
__device__ void find_request(int64_t t, const int64_t* extend_lens, int B, int* b_out,
                             int64_t* start_out) {
  const int lane = threadIdx.x & 31;
  int64_t base = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    int64_t e = b < B ? extend_lens[b] : 0;
    int64_t incl = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, b < B && base + incl > t);
    if (hit) {
      const int l = __ffs(hit) - 1;
      const int64_t excl = __shfl_sync(0xffffffffu, incl - e, l);
      *b_out = b0 + l;
      *start_out = base + excl;
      return;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  *b_out = -1;
  *start_out = 0;
}
}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads) paged_attn_simt_kernel(tf_paged_attn_args a) {
  const int64_t t = blockIdx.x;
  const int h = blockIdx.y;
  const int G = a.num_q_heads / a.num_kv_heads;
  const int D = a.head_dim;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  extern __shared__ float smem[];
  float* q_s = smem;                         // [G][D]
  float* o_s = q_s + G * D;                  // [G][D]
  float* k_s = o_s + G * D;                  // [kBK][D+1]
  float* v_s = k_s + kBK * (D + 1);          // [kBK][D]
  float* p_s = v_s + kBK * D;                // [G][kBK]
  float* m_s = p_s + G * kBK;                // [G]
  float* l_s = m_s + G;                      // [G]
  float* al_s = l_s + G;                     // [G]
  int64_t* slot_s = reinterpret_cast<int64_t*>(al_s + G + (G & 1));  // [kBK], 8-byte aligned
  __shared__ int sh_b;
  __shared__ int64_t sh_start;

  if (a.extend_lens == nullptr) {
    if (tid == 0) { sh_b = (int)t; sh_start = t; }
  } else if (warp == 0) {
    int b; int64_t st;
    find_request(t, a.extend_lens, a.batch_size, &b, &st);
    if (lane == 0) { sh_b = b; sh_start = st; }
  }
  __syncthreads();
  const int b = sh_b;
  if (b < 0) return;  // token beyond sum(extend_lens): nothing to compute
  const int64_t i = t - sh_start;
  int64_t L = a.seq_lens[b];
  if (L > a.r2t_cols) {
    if (tid == 0) record_err(a.err, TF_KERR_SLOT_RANGE);
    L = a.r2t_cols;
  }
  const int64_t E = a.extend_lens ? a.extend_lens[b] : 1;
  const int64_t q_abs = L - E + i;
  const int64_t limit = q_abs + 1 < L ? q_abs + 1 : L;  // keys j < limit are visible
  int64_t row = a.req_pool_indices[b];
  if (row < 0 || row >= a.r2t_rows) {
    if (tid == 0) record_err(a.err, TF_KERR_REQ_RANGE);
    row = 0;
  }
  const int64_t* r2t = a.req_to_token + row * a.r2t_stride;

  const T* q = reinterpret_cast<const T*>(a.q);
  for (int e = tid; e < G * D; e += kThreads) {
    const int g = e / D, d = e - (e / D) * D;
    q_s[e] = to_f(q[t * a.q_stride_tok + (int64_t)(h * G + g) * a.q_stride_head + d]);
    o_s[e] = 0.f;
  }
  if (tid < G) { m_s[tid] = -INFINITY; l_s[tid] = 0.f; }
  __syncthreads();

  const T* kb = reinterpret_cast<const T*>(a.k_buffer);
  const T* vb = reinterpret_cast<const T*>(a.v_buffer);
  for (int64_t j0 = 0; j0 < limit; j0 += kBK) {
    const int nvalid = (int)(limit - j0 < kBK ? limit - j0 : kBK);
    if (tid < nvalid) slot_s[tid] = resolve_slot(r2t[j0 + tid], a.num_slots, a.slot_mode, a.err);
    __syncthreads();
    for (int e = tid; e < nvalid * D; e += kThreads) {
      const int j = e / D, d = e - (e / D) * D;
      const int64_t off = slot_s[j] * a.kv_stride_slot + (int64_t)h * a.kv_stride_head + d;
      k_s[j * (D + 1) + d] = to_f(kb[off]);
      v_s[j * D + d] = to_f(vb[off]);
    }
    __syncthreads();
    for (int p = tid; p < G * kBK; p += kThreads) {
      const int g = p / kBK, j = p - (p / kBK) * kBK;
      float s = -INFINITY;
      if (j < nvalid) {
        float acc = 0.f;
        const float* qq = q_s + g * D;
        const float* kk = k_s + j * (D + 1);
        for (int d = 0; d < D; ++d) acc = fmaf(qq[d], kk[d], acc);
        s = acc * a.scale;
      }
      p_s[p] = s;
    }
    __syncthreads();
    for (int g = warp; g < G; g += kThreads / 32) {
      const float s = p_s[g * kBK + lane];
      const float m_old = m_s[g];
      const float m_new = fmaxf(m_old, warp_max(s));
      const float p = s == -INFINITY ? 0.f : expf(s - m_new);
      const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
      const float psum = warp_sum(p);
      p_s[g * kBK + lane] = p;
      if (lane == 0) { m_s[g] = m_new; l_s[g] = l_s[g] * alpha + psum; al_s[g] = alpha; }
    }
    __syncthreads();
    for (int e = tid; e < G * D; e += kThreads) {
      const int g = e / D, d = e - (e / D) * D;
      float acc = o_s[e] * al_s[g];
      const float* pp = p_s + g * kBK;
      for (int j = 0; j < nvalid; ++j) acc = fmaf(pp[j], v_s[j * D + d], acc);
      o_s[e] = acc;
    }
    __syncthreads();
  }

  T* out = reinterpret_cast<T*>(a.out);
  const T* gate = reinterpret_cast<const T*>(a.gate);
  for (int e = tid; e < G * D; e += kThreads) {
    const int g = e / D, d = e - (e / D) * D;
    const int hq = h * G + g;
    float o = round_to<T>(o_s[e] / l_s[g]);
    if (a.gate_mode != TF_GATE_NONE && gate != nullptr)
      o = apply_gate<T>(o, to_f(gate[t * a.gate_stride_tok + (int64_t)hq * a.gate_stride_head + d]),
                        a.gate_mode);
    out[t * a.out_stride_tok + (int64_t)hq * a.out_stride_head + d] = from_f<T>(o);
  }
}

static size_t simt_smem_bytes(int G, int D) {
  size_t floats = 2 * (size_t)G * D + kBK * (size_t)(D + 1) + kBK * (size_t)D + (size_t)G * kBK +
                  3 * (size_t)G + (G & 1);
  return floats * 4 + kBK * 8;
}

template <typename T>
static cudaError_t launch_t(const tf_paged_attn_args& a, cudaStream_t s) {
  const int G = a.num_q_heads / a.num_kv_heads;
  const size_t smem = simt_smem_bytes(G, a.head_dim);
  cudaError_t e = cudaFuncSetAttribute(paged_attn_simt_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)a.num_tokens, (unsigned)a.num_kv_heads);
  paged_attn_simt_kernel<T><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_paged_attn_simt(const tf_paged_attn_args& a, cudaStream_t s) {
  if (a.num_tokens == 0) return cudaSuccess;
  switch (a.dtype) {
    case TF_DTYPE_F32: return launch_t<float>(a, s);
    case TF_DTYPE_BF16: return launch_t<__nv_bfloat16>(a, s);
    default: return launch_t<__half>(a, s);
  }
}

}  // namespace tf
