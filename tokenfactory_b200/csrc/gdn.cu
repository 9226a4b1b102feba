// a5-a9: Gated DeltaNet (GDN) linear attention against req_to_state_pool (qwen3_8/linear_attention.py,
// qwen3_8/rms_norm_gated.py).  HBM-bound on the fp32 recurrent state.
//
// State tile layout in registers: a CTA of 2*DV threads holds one [DK x DV] fp32 state; thread
// (rg, cg) = (tid / (DV/4), tid % (DV/4)) owns rows [rg*DK/8, (rg+1)*DK/8) and the 4 columns
// [4cg, 4cg+4), so a warp reads/writes whole 512-byte row segments (float4, coalesced).  One token
// step is then
//   a_j = sum_i S_ij k_i,  c_j = sum_i S_ij q_i      (row partials in registers, 8-way smem reduce)
//   delta_j = beta (v_j - alpha a_j),  o_j = alpha c_j + delta_j (k.q)
//   S_ij <- alpha S_ij + k_i delta_j
// which is the reference's S = alpha S; v^ = S^T k; S += k (beta (v - v^))^T; o = S^T q
// (linear_attention.py:184-192, 285-297) with the products regrouped, all in fp32.
//
// decode (tf_gdn_decode): one CTA per (request, k-head) does the causal conv of the k-head's q/k
//   channels and of its v-heads' v channels (so it alone rolls those conv_state rows), then runs the
//   step for each of the Hv/Hk v-heads; the state is read once and written once per token.
// extend (tf_gdn_extend): a varlen conv kernel writes the conv outputs of every token to the
//   workspace and a second kernel rolls conv_state; the recurrent kernel then runs one CTA per
//   (request, v-head) over the request's tokens with the state resident in registers, so the state
//   costs one read and one write per request instead of per token.
#include <type_traits>

#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace tf {
namespace gdn {

template <int DK, int DV>
struct Lay {
  static constexpr int kThreads = 2 * DV;
  static constexpr int kCG = DV / 4;   // column groups (float4 each)
  static constexpr int kRG = 8;        // row groups
  static constexpr int kRPT = DK / 8;  // rows per thread
  static_assert(DK % 8 == 0 && DV % 4 == 0, "state tile");
};

// Scalars of one token for one v-head, prepared by the caller.
struct TokenScalars {
  float alpha, beta, inv_nq, inv_nk, kq;  // inv_nq includes the dk**-0.5 scale
};

struct NoHook {
  __device__ __forceinline__ void operator()() const {}
};

// One recurrent step on the register-resident state.  q_s/k_s hold RAW conv outputs (the 1/||.||
// factors are applied here), v_s the v row.  Writes o (unrounded, fp32) to o_s.  after_read() runs
// once every element of S has been consumed by the first pass (its loads have completed).
template <int DK, int DV, typename Hook = NoHook>
__device__ __forceinline__ void state_step(float4 (&S)[DK / 8], const float* q_s, const float* k_s,
                                           const float* v_s, const TokenScalars& ts, float* red_s,
                                           float* delta_s, float* o_s, Hook after_read = Hook()) {
  using Y = Lay<DK, DV>;
  const int tid = threadIdx.x;
  const int cg = tid % Y::kCG, rg = tid / Y::kCG;
  float4 pa = make_float4(0.f, 0.f, 0.f, 0.f), pc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < Y::kRPT; ++r) {
    const int i = rg * Y::kRPT + r;
    const float ki = k_s[i] * ts.inv_nk, qi = q_s[i] * ts.inv_nq;
    pa.x = fmaf(S[r].x, ki, pa.x); pa.y = fmaf(S[r].y, ki, pa.y);
    pa.z = fmaf(S[r].z, ki, pa.z); pa.w = fmaf(S[r].w, ki, pa.w);
    pc.x = fmaf(S[r].x, qi, pc.x); pc.y = fmaf(S[r].y, qi, pc.y);
    pc.z = fmaf(S[r].z, qi, pc.z); pc.w = fmaf(S[r].w, qi, pc.w);
  }
  reinterpret_cast<float4*>(red_s + (rg * 2 + 0) * DV)[cg] = pa;
  reinterpret_cast<float4*>(red_s + (rg * 2 + 1) * DV)[cg] = pc;
  after_read();
  __syncthreads();
  if (tid < DV) {
    float sa = 0.f, sc = 0.f;
#pragma unroll
    for (int g = 0; g < Y::kRG; ++g) {
      sa += red_s[(g * 2 + 0) * DV + tid];
      sc += red_s[(g * 2 + 1) * DV + tid];
    }
    const float d = ts.beta * (v_s[tid] - ts.alpha * sa);
    delta_s[tid] = d;
    o_s[tid] = fmaf(ts.alpha, sc, d * ts.kq);
  }
  __syncthreads();
  const float4 dl = reinterpret_cast<const float4*>(delta_s)[cg];
#pragma unroll
  for (int r = 0; r < Y::kRPT; ++r) {
    const int i = rg * Y::kRPT + r;
    const float ki = k_s[i] * ts.inv_nk;
    S[r].x = fmaf(ts.alpha, S[r].x, ki * dl.x);
    S[r].y = fmaf(ts.alpha, S[r].y, ki * dl.y);
    S[r].z = fmaf(ts.alpha, S[r].z, ki * dl.z);
    S[r].w = fmaf(ts.alpha, S[r].w, ki * dl.w);
  }
}

template <int DK, int DV>
__device__ __forceinline__ void load_state(float4 (&S)[DK / 8], const float* st) {
  using Y = Lay<DK, DV>;
  const int cg = threadIdx.x % Y::kCG, rg = threadIdx.x / Y::kCG;
#pragma unroll
  for (int r = 0; r < Y::kRPT; ++r)
    S[r] = __ldcs(reinterpret_cast<const float4*>(st + (size_t)(rg * Y::kRPT + r) * DV) + cg);
}

// cp.async of the state elements this thread owns into the same positions of `buf` (one group);
// take_state waits for this thread's own copies only, so neither needs a CTA barrier
template <int DK, int DV>
__device__ __forceinline__ void prefetch_state(float* buf, const float* st) {
  using Y = Lay<DK, DV>;
  const int cg = threadIdx.x % Y::kCG, rg = threadIdx.x / Y::kCG;
  const uint32_t b0 = smem_u32(buf);
#pragma unroll
  for (int r = 0; r < Y::kRPT; ++r) {
    const size_t off = (size_t)(rg * Y::kRPT + r) * DV + 4 * cg;
    cp_async16(b0 + 4 * (uint32_t)off, st + off);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int DK, int DV>
__device__ __forceinline__ void take_state(float4 (&S)[DK / 8], const float* buf) {
  using Y = Lay<DK, DV>;
  const int cg = threadIdx.x % Y::kCG, rg = threadIdx.x / Y::kCG;
  asm volatile("cp.async.wait_all;" ::: "memory");
#pragma unroll
  for (int r = 0; r < Y::kRPT; ++r)
    S[r] = reinterpret_cast<const float4*>(buf + (size_t)(rg * Y::kRPT + r) * DV)[cg];
}

template <int DK, int DV>
__device__ __forceinline__ void store_state(const float4 (&S)[DK / 8], float* st) {
  using Y = Lay<DK, DV>;
  const int cg = threadIdx.x % Y::kCG, rg = threadIdx.x / Y::kCG;
#pragma unroll
  for (int r = 0; r < Y::kRPT; ++r)
    __stcs(reinterpret_cast<float4*>(st + (size_t)(rg * Y::kRPT + r) * DV) + cg, S[r]);
}

// ||q||^2, ||k||^2 and q.k of the raw rows, one quantity per warp (round-robin); to sc_s[0..2].
template <int DK>
__device__ __forceinline__ void qk_norms(const float* q_s, const float* k_s, float* sc_s) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = (blockDim.x + 31) >> 5;
  for (int w = warp; w < 3; w += nwarps) {
    float acc = 0.f;
    for (int i = lane; i < DK; i += 32) {
      const float qv = q_s[i], kv = k_s[i];
      acc = w == 0 ? fmaf(qv, qv, acc) : (w == 1 ? fmaf(kv, kv, acc) : fmaf(qv, kv, acc));
    }
    acc = warp_sum(acc);
    if (lane == 0) sc_s[w] = acc;
  }
}

__device__ __forceinline__ TokenScalars make_scalars(const float* sc_s, float scale, float g,
                                                     float beta) {
  TokenScalars ts;
  const float nq = fmaxf(sqrtf(sc_s[0]), 1e-12f), nk = fmaxf(sqrtf(sc_s[1]), 1e-12f);
  ts.inv_nq = scale / nq;
  ts.inv_nk = 1.0f / nk;
  ts.kq = sc_s[2] * ts.inv_nq * ts.inv_nk;
  ts.alpha = expf(g);
  ts.beta = beta;
  return ts;
}

// g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b)  (linear_attention.py:178-181)
template <typename T>
__device__ __forceinline__ void gate_values(const tf_gdn_args& a, int64_t t, int vh, float* g,
                                            float* beta) {
  const float av = to_f(reinterpret_cast<const T*>(a.a)[t * a.a_stride_tok + vh]);
  const float bv = to_f(reinterpret_cast<const T*>(a.b)[t * a.b_stride_tok + vh]);
  const float al = to_f(reinterpret_cast<const T*>(a.A_log)[vh]);
  const float db = to_f(reinterpret_cast<const T*>(a.dt_bias)[vh]);
  *g = -expf(al) * softplus_f(av + db);
  *beta = 1.0f / (1.0f + expf(-bv));
}

// Output row of one v-head: o rounded to T (linear_attention.py:298), then optionally the gated
// RMSNorm w * x/rms(x) * silu(z) (rms_norm_gated.py:26-40), by warp 0.
template <typename T, int DV>
__device__ __forceinline__ void write_output(const tf_gdn_args& a, int64_t t, int vh,
                                             const float* o_s) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp != 0) return;
  T* out = reinterpret_cast<T*>(a.out) + t * a.out_stride_tok + (int64_t)vh * DV;
  constexpr int PER = (DV + 31) / 32;
  float x[PER];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int j = lane + 32 * k;
    x[k] = j < DV ? round_to<T>(o_s[j]) : 0.f;
    ss = fmaf(x[k], x[k], ss);
  }
  if (a.z == nullptr) {
#pragma unroll
    for (int k = 0; k < PER; ++k)
      if (lane + 32 * k < DV) out[lane + 32 * k] = from_f<T>(x[k]);
    return;
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)DV + a.norm_eps);
  const T* z = reinterpret_cast<const T*>(a.z) + t * a.z_stride_tok + (int64_t)vh * DV;
  const T* w = reinterpret_cast<const T*>(a.norm_weight) +
               (a.norm_weight_len == DV ? 0 : (int64_t)vh * DV);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int j = lane + 32 * k;
    if (j < DV) out[j] = from_f<T>(to_f(w[j]) * (x[k] * rs) * silu_f(to_f(z[j])));
  }
}

// write_output with silu(z) and the norm weight of the v-head already in shared memory (zs, ws:
// DV floats each; same products in the same order, so the same bits)
template <typename T, int DV>
__device__ __forceinline__ void write_output_staged(const tf_gdn_args& a, int64_t t, int vh,
                                                    const float* o_s, const float* zs,
                                                    const float* ws) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp != 0) return;
  T* out = reinterpret_cast<T*>(a.out) + t * a.out_stride_tok + (int64_t)vh * DV;
  constexpr int PER = (DV + 31) / 32;
  float x[PER];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int j = lane + 32 * k;
    x[k] = j < DV ? round_to<T>(o_s[j]) : 0.f;
    ss = fmaf(x[k], x[k], ss);
  }
  if (a.z == nullptr) {
#pragma unroll
    for (int k = 0; k < PER; ++k)
      if (lane + 32 * k < DV) out[lane + 32 * k] = from_f<T>(x[k]);
    return;
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)DV + a.norm_eps);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int j = lane + 32 * k;
    if (j < DV) out[j] = from_f<T>(ws[j] * (x[k] * rs) * zs[j]);
  }
}

// depthwise causal conv of one channel at in-request position i, then SiLU, with the reference's
// double rounding to T.  window(p) = p >= 0 ? x[p] : state[K-1+p].
template <typename T>
__device__ __forceinline__ float conv_channel(const tf_gdn_args& a, const T* xrow0, int64_t i,
                                              const T* st, int c) {
  const int K = a.conv_kernel;
  const T* w = reinterpret_cast<const T*>(a.conv_weight) + (int64_t)c * K;
  float acc = 0.f;
  for (int j = 0; j < K; ++j) {
    const int64_t p = i - (K - 1) + j;
    const float v = p >= 0 ? to_f(xrow0[p * a.qkv_stride_tok + c]) : to_f(st[c * (K - 1) + (K - 1) + p]);
    acc = fmaf(to_f(w[j]), v, acc);
  }
  if (a.conv_bias) acc += to_f(reinterpret_cast<const T*>(a.conv_bias)[c]);
  return round_to<T>(silu_f(round_to<T>(acc)));
}

// ---------------------------------------------------------------------------------------------
// decode: a persistent grid walks the (request, k-head) items
// ---------------------------------------------------------------------------------------------
// One CTA per item would leave its SM's load stream empty from its last v-head's step until the
// next CTA's first state arrives; instead each CTA takes items blockIdx.x, + gridDim.x, ... and
// keeps exactly one state in flight at all times: while v-head j of an item is stepped from
// registers, pre_s receives the next one (head j+1, or head 0 of the CTA's next item, during
// that item's conv).
template <typename T, int DK, int DV>
__global__ void __launch_bounds__(2 * DV, 2) decode_kernel(tf_gdn_args a) {
  const int Hk = a.num_k_heads;
  const int vpk = a.num_v_heads / Hk;
  const int n_items = a.batch_size * Hk;
  const int tid = threadIdx.x;
  const int key_dim = Hk * DK;
  const int K = a.conv_kernel;

  extern __shared__ float sm[];
  float* pre_s = sm;                     // [DK][DV] the state in flight
  float* q_s = sm + DK * DV;             // [DK]
  float* k_s = q_s + DK;                 // [DK]
  float* v_s = k_s + DK;                 // [vpk][DV]
  float* red_s = v_s + vpk * DV;         // [8][2][DV]
  float* delta_s = red_s + 16 * DV;      // [DV]
  float* o_s = delta_s + DV;             // [DV]
  float* sc_s = o_s + DV;                // [4]
  float* gb_s = sc_s + 4;                // [vpk][2]
  float* zs_s = gb_s + 2 * vpk;          // [vpk][DV] silu(z)
  float* ws_s = zs_s + vpk * DV;         // [vpk][DV] norm weight

  // the pool slot of item `it`, or -1 when out of range (the item is then skipped and recorded)
  auto slot_of = [&](int it) -> int64_t {
    if (it >= n_items) return -1;
    const int64_t s = a.req_pool_indices[it / Hk];
    return s >= 0 && s < a.num_slots ? s : -1;
  };
  auto state_ptr = [&](int64_t slot, int vh) -> const float* {
    return a.ssm_state + slot * a.ssm_stride_slot + (size_t)vh * DK * DV;
  };
  const float scale = rsqrtf((float)DK);
  int it = blockIdx.x;
  int64_t slot = slot_of(it);
  if (slot >= 0) prefetch_state<DK, DV>(pre_s, state_ptr(slot, (it % Hk) * vpk));
  for (; it < n_items; it += gridDim.x) {
    const int b = it / Hk, kh = it - (it / Hk) * Hk;
    const int nxt = it + gridDim.x;
    const int64_t nslot = slot_of(nxt);
    if (slot < 0) {  // nothing of this item was prefetched; start the next one's stream
      if (tid == 0) record_err(a.err, TF_KERR_REQ_RANGE);
      if (nslot >= 0) prefetch_state<DK, DV>(pre_s, state_ptr(nslot, (nxt % Hk) * vpk));
      slot = nslot;
      continue;
    }
    __syncthreads();  // the previous item's readers of q_s .. ws_s are done

    // causal conv of this item's channels; the item owns these conv_state rows
    const T* x = reinterpret_cast<const T*>(a.qkv) + (int64_t)b * a.qkv_stride_tok;
    T* cst = reinterpret_cast<T*>(a.conv_state) + slot * a.conv_stride_slot;
    const int nch = 2 * DK + vpk * DV;
    auto channel = [&](int e) {
      return e < DK ? kh * DK + e
                    : (e < 2 * DK ? key_dim + kh * DK + (e - DK) : 2 * key_dim + kh * vpk * DV + (e - 2 * DK));
    };
    const T* zr = a.z ? reinterpret_cast<const T*>(a.z) + (int64_t)b * a.z_stride_tok + (int64_t)kh * vpk * DV
                      : nullptr;
    const bool shared_w = a.norm_weight_len == DV;
    const T* wr = a.z ? reinterpret_cast<const T*>(a.norm_weight) + (shared_w ? 0 : (int64_t)kh * vpk * DV)
                      : nullptr;
    const int bdim = blockDim.x;
    if (sizeof(T) == 2 && K == 4 && nch <= 3 * bdim && vpk * DV <= 2 * bdim &&
        (reinterpret_cast<uintptr_t>(a.conv_weight) & 7) == 0) {
      // 16-bit activations (a channel's 4 weights are one 8-byte load): every load of the item
      // first (conv windows, weights and inputs of up to 3 channels per thread, z and the norm
      // weights, the gates), then the arithmetic: one memory round trip
      // instead of one per pass.  Same products and roundings as the loop below.
      T st[3][3], xv[3], zv[2], wv2[2];
      uint2 w4[3];
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int e = tid + u * bdim;
        if (e < nch) {
          const int c = channel(e);
          const T* sp = cst + (int64_t)c * 3;
          st[u][0] = sp[0];
          st[u][1] = sp[1];
          st[u][2] = sp[2];
          xv[u] = x[c];
          w4[u] = *reinterpret_cast<const uint2*>(reinterpret_cast<const T*>(a.conv_weight) + (int64_t)c * 4);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int e = tid + u * bdim;
        if (zr != nullptr && e < vpk * DV) {
          zv[u] = zr[e];
          wv2[u] = wr[shared_w ? e % DV : e];
        }
      }
      if (tid < vpk) {
        float g, be;
        gate_values<T>(a, b, kh * vpk + tid, &g, &be);
        gb_s[2 * tid] = g;
        gb_s[2 * tid + 1] = be;
      }
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int e = tid + u * bdim;
        if (e < nch) {
          const T* wt = reinterpret_cast<const T*>(&w4[u]);
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < 3; ++j) acc = fmaf(to_f(wt[j]), to_f(st[u][j]), acc);
          acc = fmaf(to_f(wt[3]), to_f(xv[u]), acc);
          const int c = channel(e);
          if (a.conv_bias) acc += to_f(reinterpret_cast<const T*>(a.conv_bias)[c]);
          T* sp = cst + (int64_t)c * 3;
          sp[0] = st[u][1];
          sp[1] = st[u][2];
          sp[2] = xv[u];
          q_s[e] = round_to<T>(silu_f(round_to<T>(acc)));  // q_s | k_s | v_s are contiguous
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int e = tid + u * bdim;
        if (zr != nullptr && e < vpk * DV) {
          zs_s[e] = silu_f(to_f(zv[u]));
          ws_s[e] = to_f(wv2[u]);
        }
      }
    } else {
      for (int e = tid; e < nch; e += bdim) {
        const int c = channel(e);
        float win[8];
        for (int j = 0; j < K - 1; ++j) win[j] = to_f(cst[(int64_t)c * (K - 1) + j]);
        const float xvf = to_f(x[c]);
        const T* w = reinterpret_cast<const T*>(a.conv_weight) + (int64_t)c * K;
        float acc = 0.f;
        for (int j = 0; j < K - 1; ++j) acc = fmaf(to_f(w[j]), win[j], acc);
        acc = fmaf(to_f(w[K - 1]), xvf, acc);
        if (a.conv_bias) acc += to_f(reinterpret_cast<const T*>(a.conv_bias)[c]);
        const float y = round_to<T>(silu_f(round_to<T>(acc)));
        for (int j = 0; j + 1 < K - 1; ++j) cst[(int64_t)c * (K - 1) + j] = from_f<T>(win[j + 1]);
        if (K > 1) cst[(int64_t)c * (K - 1) + K - 2] = x[c];
        q_s[e] = y;  // q_s | k_s | v_s are contiguous
      }
      if (tid < vpk) {
        float g, be;
        gate_values<T>(a, b, kh * vpk + tid, &g, &be);
        gb_s[2 * tid] = g;
        gb_s[2 * tid + 1] = be;
      }
      if (zr != nullptr) {  // the output gate's operands, off the per-head critical path
        for (int e = tid; e < vpk * DV; e += bdim) {
          zs_s[e] = silu_f(to_f(zr[e]));
          ws_s[e] = to_f(wr[shared_w ? e % DV : e]);
        }
      }
    }
    __syncthreads();
    qk_norms<DK>(q_s, k_s, sc_s);
    __syncthreads();
    // No barrier closes a v-head: red_s and delta_s of head j+1 are written only after the first
    // barrier of its step, which every thread reaches after its last read of head j's, and warp 0
    // reads o_s (write_output_staged) before it reaches that barrier.
    for (int j = 0; j < vpk; ++j) {
      const int vh = kh * vpk + j;
      float4 S[DK / 8];
      take_state<DK, DV>(S, pre_s);
      // the next state is requested once this thread's reads of pre_s have been consumed
      const float* next = j + 1 < vpk ? state_ptr(slot, vh + 1)
                                      : (nslot >= 0 ? state_ptr(nslot, (nxt % Hk) * vpk) : nullptr);
      auto refill = [&]() {
        if (next != nullptr) prefetch_state<DK, DV>(pre_s, next);
      };
      const TokenScalars ts = make_scalars(sc_s, scale, gb_s[2 * j], gb_s[2 * j + 1]);
      state_step<DK, DV>(S, q_s, k_s, v_s + j * DV, ts, red_s, delta_s, o_s, refill);
      store_state<DK, DV>(S, a.ssm_state + slot * a.ssm_stride_slot + (size_t)vh * DK * DV);
      write_output_staged<T, DV>(a, b, vh, o_s, zs_s + j * DV, ws_s + j * DV);
    }
    slot = nslot;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // nothing in flight into shared memory at exit
}

// ---------------------------------------------------------------------------------------------
// extend: conv over every token (varlen), conv_state roll, recurrent kernel per (request, v-head)
// ---------------------------------------------------------------------------------------------
// token t -> request b and its first token, by one warp
__device__ void find_request(int64_t t, const int64_t* ext, int B, int* b_out, int64_t* start_out) {
  const int lane = threadIdx.x & 31;
  int64_t base = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int64_t e = b < B ? ext[b] : 0;
    int64_t incl = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, b < B && base + incl > t);
    if (hit) {
      const int l = __ffs(hit) - 1;
      *b_out = b0 + l;
      *start_out = base + __shfl_sync(0xffffffffu, incl - e, l);
      return;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  *b_out = -1;
  *start_out = 0;
}

// extend_len of request b, cut to the tokens the batch holds (a longer one is recorded)
__device__ __forceinline__ int64_t clamp_extend(const tf_gdn_args& a, int b, int64_t t0) {
  const int64_t E = a.extend_lens[b];
  if (t0 + E > a.num_tokens) {
    record_err(a.err, TF_KERR_REQ_RANGE);
    return a.num_tokens - t0 > 0 ? a.num_tokens - t0 : 0;
  }
  return E;
}

// token offsets of every request (exclusive prefix of extend_lens), one CTA
__global__ void offsets_kernel(const int64_t* ext, int B, int64_t* start) {
  if (threadIdx.x == 0) {
    int64_t s = 0;
    for (int b = 0; b < B; ++b) { start[b] = s; s += ext[b]; }
    start[B] = s;
  }
}

// order[k] = the request with the k-th longest extend (ties by index): the chunk kernel takes its
// CTAs longest request first, so that the longest chains do not start last (scheduling only)
__global__ void order_kernel(const int64_t* ext, int B, int32_t* order) {
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int64_t e = ext[b];
    int rank = 0;
    for (int o = 0; o < B; ++o) {
      const int64_t eo = ext[o];
      rank += (eo > e) || (eo == e && o < b);
    }
    order[rank] = b;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) conv_extend_kernel(tf_gdn_args a, const int64_t* start,
                                                          T* conv_out) {
  const int64_t t = blockIdx.x;
  __shared__ int sb;
  if (threadIdx.x < 32) {
    int b; int64_t st;
    find_request(t, a.extend_lens, a.batch_size, &b, &st);
    if (threadIdx.x == 0) sb = b;
  }
  __syncthreads();
  const int b = sb;
  if (b < 0) return;
  const int64_t slot = a.req_pool_indices[b];
  if (slot < 0 || slot >= a.num_slots) {
    if (threadIdx.x == 0) record_err(a.err, TF_KERR_REQ_RANGE);
    return;
  }
  const int conv_dim = 2 * a.num_k_heads * a.head_k_dim + a.num_v_heads * a.head_v_dim;
  const T* x0 = reinterpret_cast<const T*>(a.qkv) + start[b] * a.qkv_stride_tok;
  const T* st = reinterpret_cast<const T*>(a.conv_state) + slot * a.conv_stride_slot;
  const int64_t i = t - start[b];
  for (int c = threadIdx.x; c < conv_dim; c += blockDim.x)
    conv_out[t * conv_dim + c] = from_f<T>(conv_channel<T>(a, x0, i, st, c));
}

// Same conv for K = 4, tiled: one CTA per (64-token chunk of the packed batch, 512 channels); a
// thread owns two adjacent channels, keeps their weights and the last three inputs of the current
// request in registers and walks the chunk's tokens, reloading the window from conv_state (or from
// the preceding tokens) where a request starts.  Every input element is read once.
template <typename T>
__device__ __forceinline__ void load_pair(const T* p, bool vec, float& x0, float& x1) {
  if constexpr (sizeof(T) == 2) {
    if (vec) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
      const T* h = reinterpret_cast<const T*>(&w);
      x0 = to_f(h[0]);
      x1 = to_f(h[1]);
      return;
    }
  }
  x0 = to_f(p[0]);
  x1 = to_f(p[1]);
}

constexpr int kConvTok = 64;
constexpr int kConvThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kConvThreads) conv4_tiled_kernel(tf_gdn_args a, const int64_t* start,
                                                                   T* conv_out) {
  const int conv_dim = 2 * a.num_k_heads * a.head_k_dim + a.num_v_heads * a.head_v_dim;
  const int c = (blockIdx.x * kConvThreads + threadIdx.x) * 2;
  const int64_t T_all = start[a.batch_size] < a.num_tokens ? start[a.batch_size] : a.num_tokens;
  const int64_t t_begin = (int64_t)blockIdx.y * kConvTok;
  if (t_begin >= T_all) return;
  const int64_t t_end = t_begin + kConvTok < T_all ? t_begin + kConvTok : T_all;
  // request of the chunk's first token: binary search over start[0..B]
  __shared__ int s_b;
  if (threadIdx.x == 0) {
    int lo = 0, hi = a.batch_size - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] <= t_begin) lo = mid; else hi = mid - 1;
    }
    s_b = lo;
  }
  __syncthreads();
  if (c >= conv_dim) return;
  const T* wt = reinterpret_cast<const T*>(a.conv_weight);
  float w0[4], w1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    w0[j] = to_f(wt[(int64_t)c * 4 + j]);
    w1[j] = to_f(wt[(int64_t)(c + 1) * 4 + j]);
  }
  const T* cb = reinterpret_cast<const T*>(a.conv_bias);
  const float b0 = cb ? to_f(cb[c]) : 0.f, b1 = cb ? to_f(cb[c + 1]) : 0.f;
  const T* x = reinterpret_cast<const T*>(a.qkv);
  const bool xvec = ((reinterpret_cast<uintptr_t>(x) & 3) == 0) && (a.qkv_stride_tok % 2 == 0);
  int b = s_b;
  int64_t rs = start[b], re = start[b + 1];
  float h0[3], h1[3];  // inputs at positions i-3, i-2, i-1 of the current request
  bool need_init = true;
  for (int64_t t = t_begin; t < t_end; ++t) {
    while (t >= re) {  // next request (uniform over the CTA)
      ++b;
      rs = re;
      re = start[b + 1];
      need_init = true;
    }
    if (need_init) {
      const int64_t slot = a.req_pool_indices[b];
      const bool ok = slot >= 0 && slot < a.num_slots;
      const T* st = reinterpret_cast<const T*>(a.conv_state) + (ok ? slot : 0) * a.conv_stride_slot;
      const int64_t i = t - rs;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int64_t p = i - 3 + j;
        if (p >= 0) {
          load_pair<T>(x + (rs + p) * a.qkv_stride_tok + c, xvec, h0[j], h1[j]);
        } else {
          h0[j] = ok ? to_f(st[(int64_t)c * 3 + 3 + p]) : 0.f;
          h1[j] = ok ? to_f(st[(int64_t)(c + 1) * 3 + 3 + p]) : 0.f;
        }
      }
      if (!ok && c == 0) record_err(a.err, TF_KERR_REQ_RANGE);
      need_init = false;
    }
    float x0, x1;
    load_pair<T>(x + t * a.qkv_stride_tok + c, xvec, x0, x1);
    float acc0 = fmaf(w0[0], h0[0], fmaf(w0[1], h0[1], fmaf(w0[2], h0[2], fmaf(w0[3], x0, b0))));
    float acc1 = fmaf(w1[0], h1[0], fmaf(w1[1], h1[1], fmaf(w1[2], h1[2], fmaf(w1[3], x1, b1))));
    acc0 = round_to<T>(silu_f(round_to<T>(acc0)));
    acc1 = round_to<T>(silu_f(round_to<T>(acc1)));
    T* o = conv_out + t * conv_dim + c;
    if constexpr (sizeof(T) == 2) {
      T pr[2] = {from_f<T>(acc0), from_f<T>(acc1)};
      *reinterpret_cast<uint32_t*>(o) = *reinterpret_cast<uint32_t*>(pr);
    } else {
      o[0] = from_f<T>(acc0);
      o[1] = from_f<T>(acc1);
    }
    h0[0] = h0[1]; h0[1] = h0[2]; h0[2] = x0;
    h1[0] = h1[1]; h1[1] = h1[2]; h1[2] = x1;
  }
}

// K = 4 conv for 16-bit activations with 8-byte rows (4 channels per thread).  Same FMA order and
// roundings as conv4_tiled_kernel; SiLU with a hardware exponential and an approximate division
// (the result is rounded to the 16-bit type, where the two differ in rare last-place cases).
constexpr int kConvVecTok = 8;
constexpr int kConvVecThreads = 128;

__device__ __forceinline__ float silu_rt(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Sliding window: a thread takes 4 channels of kConvPipeBlocks consecutive 8-token blocks.  The
// next block's 8 new rows are requested before the current block is computed (the 3 rows before
// them are the current window's last), so every warp keeps loads in flight while it computes, and
// each row is loaded once per thread (one 11-row window per block measured 240 us against 215 us
// at config 4).
constexpr int kConvPipeBlocks = 8;

template <typename T>
__global__ void __launch_bounds__(kConvVecThreads, 5) conv4_pipe_kernel(tf_gdn_args a,
                                                                        const int64_t* start,
                                                                        T* conv_out) {
  static_assert(sizeof(T) == 2, "16-bit activations");
  const int conv_dim = 2 * a.num_k_heads * a.head_k_dim + a.num_v_heads * a.head_v_dim;
  const int c = (blockIdx.x * kConvVecThreads + threadIdx.x) * 4;
  if (c >= conv_dim) return;  // no barrier in this kernel
  const int64_t T_all = start[a.batch_size] < a.num_tokens ? start[a.batch_size] : a.num_tokens;
  const int64_t t0 = (int64_t)blockIdx.y * (kConvVecTok * kConvPipeBlocks);
  if (t0 >= T_all) return;
  const T* x = reinterpret_cast<const T*>(a.qkv) + c;
  auto row = [&](int64_t t) -> uint2 {
    return (t >= 0 && t < T_all) ? __ldcs(reinterpret_cast<const uint2*>(x + t * a.qkv_stride_tok))
                                 : make_uint2(0u, 0u);
  };
  uint2 win[kConvVecTok + 3];  // rows tb-3 .. tb+7 of the current block
#pragma unroll
  for (int r = 0; r < kConvVecTok + 3; ++r) win[r] = row(t0 - 3 + r);
  float w[4][4], bias[4];
  const T* wt = reinterpret_cast<const T*>(a.conv_weight) + (int64_t)c * 4;
  const T* cb = reinterpret_cast<const T*>(a.conv_bias);
  if ((reinterpret_cast<uintptr_t>(a.conv_weight) & 15) == 0) {  // 4 channels x 4 taps: 32 bytes
    const uint4 w01 = __ldg(reinterpret_cast<const uint4*>(wt));
    const uint4 w23 = __ldg(reinterpret_cast<const uint4*>(wt) + 1);
    const uint32_t wv[8] = {w01.x, w01.y, w01.z, w01.w, w23.x, w23.y, w23.z, w23.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      w[e][0] = unpack_lo<T>(wv[2 * e]);
      w[e][1] = unpack_hi<T>(wv[2 * e]);
      w[e][2] = unpack_lo<T>(wv[2 * e + 1]);
      w[e][3] = unpack_hi<T>(wv[2 * e + 1]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int j = 0; j < 4; ++j) w[e][j] = to_f(wt[e * 4 + j]);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) bias[e] = cb ? to_f(cb[c + e]) : 0.f;
  int b;  // request of the first token (start[] is small and stays in cache)
  {
    int lo = 0, hi = a.batch_size - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] <= t0) lo = mid; else hi = mid - 1;
    }
    b = lo;
  }
  int64_t rs = start[b], re = start[b + 1];
#pragma unroll 1
  for (int k = 0; k < kConvPipeBlocks; ++k) {
    const int64_t tb = t0 + (int64_t)k * kConvVecTok;
    if (tb >= T_all) break;
    uint2 nxt[kConvVecTok];  // the next block's new rows, in flight while this block computes
    const bool more = k + 1 < kConvPipeBlocks;
#pragma unroll
    for (int r = 0; r < kConvVecTok; ++r) nxt[r] = more ? row(tb + kConvVecTok + r) : make_uint2(0u, 0u);
#pragma unroll
    for (int i = 0; i < kConvVecTok; ++i) {
      const int64_t t = tb + i;
      if (t >= T_all) break;
      while (t >= re) {  // next request
        ++b;
        rs = re;
        re = start[b + 1];
      }
      float h[3][4];
#pragma unroll
      for (int q = 0; q < 3; ++q) {  // history rows t-3+q
        const T* hv = reinterpret_cast<const T*>(&win[i + q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[q][e] = to_f(hv[e]);
      }
      if (t - rs < 3) {  // the first tokens of a request read its conv_state
        const int64_t slot = a.req_pool_indices[b];
        const bool ok = slot >= 0 && slot < a.num_slots;
        if (!ok && c == 0) record_err(a.err, TF_KERR_REQ_RANGE);
        const T* st = reinterpret_cast<const T*>(a.conv_state) + (ok ? slot : 0) * a.conv_stride_slot;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          const int64_t p = t - rs - 3 + q;  // position inside the request
          if (p < 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) h[q][e] = ok ? to_f(st[(int64_t)(c + e) * 3 + 3 + p]) : 0.f;
          }
        }
      }
      const T* xv = reinterpret_cast<const T*>(&win[i + 3]);
      float acc[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        acc[e] = fmaf(w[e][0], h[0][e], fmaf(w[e][1], h[1][e],
                      fmaf(w[e][2], h[2][e], fmaf(w[e][3], to_f(xv[e]), bias[e]))));
      uint32_t ow[2];
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const uint32_t r = pack2_rn<T>(acc[2 * e2], acc[2 * e2 + 1]);
        ow[e2] = pack2_rn<T>(silu_rt(unpack_lo<T>(r)), silu_rt(unpack_hi<T>(r)));
      }
      __stcs(reinterpret_cast<uint2*>(conv_out + t * conv_dim + c), make_uint2(ow[0], ow[1]));
    }
#pragma unroll
    for (int r = 0; r < 3; ++r) win[r] = win[kConvVecTok + r];
#pragma unroll
    for (int r = 0; r < kConvVecTok; ++r) win[3 + r] = nxt[r];
  }
}

// conv_state <- last K-1 columns of [state | x] per (request, channel)  (linear_attention.py:142-143)
template <typename T>
__global__ void conv_state_roll_kernel(tf_gdn_args a, const int64_t* start) {
  const int b = blockIdx.y;
  const int conv_dim = 2 * a.num_k_heads * a.head_k_dim + a.num_v_heads * a.head_v_dim;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= conv_dim) return;
  const int64_t slot = a.req_pool_indices[b];
  if (slot < 0 || slot >= a.num_slots) return;
  const int K = a.conv_kernel;
  const int64_t E = clamp_extend(a, b, start[b]);
  T* st = reinterpret_cast<T*>(a.conv_state) + slot * a.conv_stride_slot + (int64_t)c * (K - 1);
  const T* x0 = reinterpret_cast<const T*>(a.qkv) + start[b] * a.qkv_stride_tok + c;
  T nw[8];
  for (int k = 0; k < K - 1; ++k) {
    const int64_t p = E + k;  // index into padded = [state(K-1) | x(E)]
    nw[k] = p < K - 1 ? st[p] : x0[(p - (K - 1)) * a.qkv_stride_tok];
  }
  for (int k = 0; k < K - 1; ++k) st[k] = nw[k];
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(2 * DV) recurrent_extend_kernel(tf_gdn_args a,
                                                                  const int64_t* start,
                                                                  const T* conv_out) {
  const int b = blockIdx.x / a.num_v_heads;
  const int vh = blockIdx.x - b * a.num_v_heads;
  const int vpk = a.num_v_heads / a.num_k_heads;
  const int kh = vh / vpk;
  const int tid = threadIdx.x;
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * DV;

  extern __shared__ float sm[];
  float* q_s = sm;                  // [DK]
  float* k_s = q_s + DK;            // [DK]
  float* v_s = k_s + DK;            // [DV]
  float* red_s = v_s + DV;          // [8][2][DV]
  float* delta_s = red_s + 16 * DV; // [DV]
  float* o_s = delta_s + DV;        // [DV]
  float* sc_s = o_s + DV;           // [4]
  float* gb_s = sc_s + 4;           // [2]

  const int64_t slot = a.req_pool_indices[b];
  if (slot < 0 || slot >= a.num_slots) return;  // recorded by the conv kernel
  const int64_t t0 = start[b];
  const int64_t E = clamp_extend(a, b, t0);
  if (E <= 0) return;
  float* st = a.ssm_state + slot * a.ssm_stride_slot + (size_t)vh * DK * DV;
  float4 S[DK / 8];
  load_state<DK, DV>(S, st);
  const float scale = rsqrtf((float)DK);
  for (int64_t i = 0; i < E; ++i) {
    const int64_t t = t0 + i;
    const T* row = conv_out + t * conv_dim;
    for (int e = tid; e < 2 * DK + DV; e += blockDim.x) {
      int c;
      if (e < DK) c = kh * DK + e;
      else if (e < 2 * DK) c = key_dim + kh * DK + (e - DK);
      else c = 2 * key_dim + vh * DV + (e - 2 * DK);
      sm[e] = to_f(row[c]);
    }
    if (tid == 0) gate_values<T>(a, t, vh, &gb_s[0], &gb_s[1]);
    __syncthreads();
    qk_norms<DK>(q_s, k_s, sc_s);
    __syncthreads();
    const TokenScalars ts = make_scalars(sc_s, scale, gb_s[0], gb_s[1]);
    state_step<DK, DV>(S, q_s, k_s, v_s, ts, red_s, delta_s, o_s);
    write_output<T, DV>(a, t, vh, o_s);
    __syncthreads();
  }
  store_state<DK, DV>(S, st);
}

// ---------------------------------------------------------------------------------------------
// a7: chunked gated delta rule (qwen3_8/linear_attention.py:194-240), one CTA per (request, v-head)
// over the request's tokens in chunks of C = 64, everything in fp32 on CUDA cores (the reference is
// fp32 end to end; the state products keep full fp32 precision).  Per chunk, with gamma the in-chunk
// cumulative log decay:
//   Mk = strict_tril(beta_i e^(gamma_i - gamma_j)) o K K^T,  Mq = tril(e^(gamma_i - gamma_j)) o Q K^T
//   U  = beta (V - e^gamma K S)            then  (I + Mk) U' = U   (forward substitution)
//   O  = e^gamma Q S + Mq U'
//   S  = e^gamma_C S + (K o e^(gamma_C - gamma))^T U'
// The state, the chunk's Q/K/U rows and the two C x C matrices live in shared memory with padded
// rows (float4 accesses stay conflict-free); the output goes through the fused gated RMSNorm.
// ---------------------------------------------------------------------------------------------
template <int D>
struct ChunkLay {
  static constexpr int C = 64;
  static constexpr int kThreads = 256;
  static constexpr int P = D + 4;        // row pitch of [*, D] tiles, floats
  static constexpr int MP = C + 4;       // row pitch of the C x C tiles
  static constexpr int oS = 0;           // state [D][P]
  static constexpr int oQ = oS + D * P;  // Q rows, then O rows [C][P]
  static constexpr int oK = oQ + C * P;  // K rows [C][P]
  static constexpr int oU = oK + C * P;  // V -> rhs -> U' rows [C][P]
  static constexpr int oMk = oU + C * P; // [C][MP]
  static constexpr int oMq = oMk + C * MP;
  static constexpr int oG = oMq + C * MP;  // gamma [C]
  static constexpr int oB = oG + C;        // beta [C]
  static constexpr int oEnd = oB + C;
  static constexpr size_t kBytes = (size_t)oEnd * 4;
  static constexpr int NCG = D / 4;            // float4 column groups
  static constexpr int NRG = kThreads / NCG;   // row groups
  static_assert(kThreads % NCG == 0 && C % NRG == 0 && D % NRG == 0, "chunk tiling");
};

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void sts4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
}

template <typename T, int D>
__global__ void __launch_bounds__(256, 1) chunk_extend_kernel(tf_gdn_args a, const int64_t* start,
                                                              const T* conv_out) {
  using Y = ChunkLay<D>;
  constexpr int C = Y::C, P = Y::P, MP = Y::MP, NCG = Y::NCG, NRG = Y::NRG;
  const int b = blockIdx.x / a.num_v_heads;
  const int vh = blockIdx.x - b * a.num_v_heads;
  const int vpk = a.num_v_heads / a.num_k_heads;
  const int kh = vh / vpk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int key_dim = a.num_k_heads * D;
  const int conv_dim = 2 * key_dim + a.num_v_heads * D;

  extern __shared__ float4 sm4[];
  float* sm = reinterpret_cast<float*>(sm4);
  float* Ss = sm + Y::oS;
  float* Qs = sm + Y::oQ;
  float* Ks = sm + Y::oK;
  float* Us = sm + Y::oU;
  float* Mk = sm + Y::oMk;
  float* Mq = sm + Y::oMq;
  float* gam = sm + Y::oG;
  float* bet = sm + Y::oB;

  const int64_t slot = a.req_pool_indices[b];
  if (slot < 0 || slot >= a.num_slots) return;  // recorded by the conv kernel
  const int64_t t0 = start[b];
  const int64_t E = clamp_extend(a, b, t0);
  if (E <= 0) return;
  float* st = a.ssm_state + slot * a.ssm_stride_slot + (size_t)vh * D * D;
  for (int e = tid; e < D * NCG; e += Y::kThreads) {
    const int r = e / NCG, cg = e - (e / NCG) * NCG;
    sts4(Ss + r * P + 4 * cg, __ldcs(reinterpret_cast<const float4*>(st + (size_t)r * D) + cg));
  }
  const float qscale = rsqrtf((float)D);
  const int rg = tid / NCG, cg = tid - (tid / NCG) * NCG;

  for (int64_t c0 = 0; c0 < E; c0 += C) {
    const int c = (int)(E - c0 < C ? E - c0 : C);
    // ---- load the chunk: raw q, k, v rows into shared memory (every load in flight at once),
    // g and beta of token t by thread t; then each warp normalises whole q / k rows in place
    {
      constexpr int EPV = 16 / (int)sizeof(T);        // elements per 16-byte load
      constexpr int VPR = D / EPV;                     // vectors per row part
      constexpr int NV = C * 3 * VPR / Y::kThreads;    // vectors per thread
      static_assert(C * 3 * VPR % Y::kThreads == 0, "load tiling");
      uint4 raw[NV];
#pragma unroll
      for (int n = 0; n < NV; ++n) {  // all loads of the chunk in flight before any use
        const int e = tid + n * Y::kThreads;
        const int i = e / (3 * VPR), rem = e - (e / (3 * VPR)) * (3 * VPR);
        const int part = rem / VPR, vi = rem - (rem / VPR) * VPR;
        const int col = part == 0 ? kh * D : (part == 1 ? key_dim + kh * D : 2 * key_dim + vh * D);
        raw[n] = i < c ? *reinterpret_cast<const uint4*>(conv_out + (t0 + c0 + i) * conv_dim + col + vi * EPV)
                       : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int n = 0; n < NV; ++n) {
        const int e = tid + n * Y::kThreads;
        const int i = e / (3 * VPR), rem = e - (e / (3 * VPR)) * (3 * VPR);
        const int part = rem / VPR, vi = rem - (rem / VPR) * VPR;
        float* dst = (part == 0 ? Qs : (part == 1 ? Ks : Us)) + i * P + vi * EPV;
        const T* src = reinterpret_cast<const T*>(&raw[n]);
#pragma unroll
        for (int q = 0; q < EPV; ++q) dst[q] = to_f(src[q]);
      }
    }
    if (tid < C) {
      float g = 0.f, be = 0.f;
      if (tid < c) gate_values<T>(a, t0 + c0 + tid, vh, &g, &be);
      gam[tid] = g;
      bet[tid] = be;
    }
    __syncthreads();
    for (int i = warp; i < c; i += Y::kThreads / 32) {
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int k = 0; k < D / 32; ++k) {
        const float qv = Qs[i * P + lane + 32 * k], kv = Ks[i * P + lane + 32 * k];
        sq = fmaf(qv, qv, sq);
        sk = fmaf(kv, kv, sk);
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      const float iq = qscale / fmaxf(sqrtf(sq), 1e-12f), ik = 1.0f / fmaxf(sqrtf(sk), 1e-12f);
#pragma unroll
      for (int k = 0; k < D / 32; ++k) {
        Qs[i * P + lane + 32 * k] *= iq;
        Ks[i * P + lane + 32 * k] *= ik;
      }
    }
    if (warp == 0) {  // gamma = inclusive cumulative sum of g over the chunk
      float g0 = gam[2 * lane], g1 = gam[2 * lane + 1];
      float incl = g0 + g1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const float excl = incl - (g0 + g1);
      gam[2 * lane] = excl + g0;
      gam[2 * lane + 1] = incl;
    }
    __syncthreads();

    // ---- Mk = strict_tril(beta_i e^(gi-gj)) K K^T,  Mq = tril(e^(gi-gj)) Q K^T
    {
      const int ti = tid >> 4, tj = tid & 15;
      float ak[4][4], aq[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) ak[r][s2] = aq[r][s2] = 0.f;
#pragma unroll 2
      for (int d = 0; d < D; d += 4) {
        float4 kr[4], qr[4], kc[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          kr[r] = lds4(Ks + (ti + 16 * r) * P + d);
          qr[r] = lds4(Qs + (ti + 16 * r) * P + d);
          kc[r] = lds4(Ks + (tj + 16 * r) * P + d);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int s2 = 0; s2 < 4; ++s2) {
            ak[r][s2] = dot4(kr[r], kc[s2], ak[r][s2]);
            aq[r][s2] = dot4(qr[r], kc[s2], aq[r][s2]);
          }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = ti + 16 * r;
        const float gi = gam[i], bi = bet[i];
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
          const int j = tj + 16 * s2;
          const float dec = j <= i ? expf(gi - gam[j]) : 0.f;
          Mk[i * MP + j] = j < i ? bi * dec * ak[r][s2] : 0.f;
          Mq[i * MP + j] = dec * aq[r][s2];
        }
      }
    }
    // ---- K S and Q S for rows [rg*C/NRG, ...): rhs into U, e^gamma Q S into the Q rows
    {
      constexpr int RPT = C / NRG;
      float4 aks[RPT], aqs[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) aks[r] = aqs[r] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int i0 = rg * RPT;
#pragma unroll 1
      for (int d = 0; d < D; d += 4) {
        const float4 s0 = lds4(Ss + (d + 0) * P + 4 * cg), s1 = lds4(Ss + (d + 1) * P + 4 * cg);
        const float4 s2v = lds4(Ss + (d + 2) * P + 4 * cg), s3 = lds4(Ss + (d + 3) * P + 4 * cg);
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
          const float4 kk = lds4(Ks + (i0 + r) * P + d), qq = lds4(Qs + (i0 + r) * P + d);
          aks[r].x = fmaf(kk.x, s0.x, fmaf(kk.y, s1.x, fmaf(kk.z, s2v.x, fmaf(kk.w, s3.x, aks[r].x))));
          aks[r].y = fmaf(kk.x, s0.y, fmaf(kk.y, s1.y, fmaf(kk.z, s2v.y, fmaf(kk.w, s3.y, aks[r].y))));
          aks[r].z = fmaf(kk.x, s0.z, fmaf(kk.y, s1.z, fmaf(kk.z, s2v.z, fmaf(kk.w, s3.z, aks[r].z))));
          aks[r].w = fmaf(kk.x, s0.w, fmaf(kk.y, s1.w, fmaf(kk.z, s2v.w, fmaf(kk.w, s3.w, aks[r].w))));
          aqs[r].x = fmaf(qq.x, s0.x, fmaf(qq.y, s1.x, fmaf(qq.z, s2v.x, fmaf(qq.w, s3.x, aqs[r].x))));
          aqs[r].y = fmaf(qq.x, s0.y, fmaf(qq.y, s1.y, fmaf(qq.z, s2v.y, fmaf(qq.w, s3.y, aqs[r].y))));
          aqs[r].z = fmaf(qq.x, s0.z, fmaf(qq.y, s1.z, fmaf(qq.z, s2v.z, fmaf(qq.w, s3.z, aqs[r].z))));
          aqs[r].w = fmaf(qq.x, s0.w, fmaf(qq.y, s1.w, fmaf(qq.z, s2v.w, fmaf(qq.w, s3.w, aqs[r].w))));
        }
      }
      __syncthreads();  // every thread is done reading Q before its rows are overwritten with O
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int i = i0 + r;
        const float eg = expf(gam[i]), bi = bet[i];
        float4 u = lds4(Us + i * P + 4 * cg);
        u.x = bi * (u.x - eg * aks[r].x);
        u.y = bi * (u.y - eg * aks[r].y);
        u.z = bi * (u.z - eg * aks[r].z);
        u.w = bi * (u.w - eg * aks[r].w);
        sts4(Us + i * P + 4 * cg, u);
        sts4(Qs + i * P + 4 * cg, make_float4(eg * aqs[r].x, eg * aqs[r].y, eg * aqs[r].z, eg * aqs[r].w));
      }
    }
    __syncthreads();
    // ---- (I + Mk) U' = U: forward substitution.  Two lanes per column; lane parity p keeps rows
    // j = 2m + p of its column in registers.  Mk is strictly lower triangular, so both parities
    // sum over the same compile-time range of m (the entries with j >= i are zero).
    if (c > 1) {
      const int col = tid >> 1, par = tid & 1;
      const bool has_col = col < D;  // D = 64: warps 4-7 only keep the shuffles matched
      float ur[C / 2];
#pragma unroll
      for (int m = 0; m < C / 2; ++m) ur[m] = has_col ? Us[(2 * m + par) * P + col] : 0.f;
#pragma unroll
      for (int i = 1; i < C; ++i) {
        float acc0 = 0.f, acc1 = 0.f;
        const float* mrow = Mk + i * MP + par;
#pragma unroll
        for (int m = 0; m < (i + 1) / 2; ++m) {
          if (m & 1) acc1 = fmaf(mrow[2 * m], ur[m], acc1);
          else acc0 = fmaf(mrow[2 * m], ur[m], acc0);
        }
        float acc = acc0 + acc1;
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        if (par == (i & 1)) ur[i >> 1] -= acc;
      }
      __syncwarp();
      if (has_col) {
#pragma unroll
        for (int m = 0; m < C / 2; ++m) Us[(2 * m + par) * P + col] = ur[m];
      }
    }
    __syncthreads();
    // ---- O += Mq U'  and  S = e^gC S + (K o e^(gC - g))^T U'
    {
      constexpr int RPT = C / NRG;
      const int i0 = rg * RPT;
      float4 ao[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) ao[r] = lds4(Qs + (i0 + r) * P + 4 * cg);
#pragma unroll 1
      for (int j = 0; j < C; j += 4) {
        const float4 u0 = lds4(Us + (j + 0) * P + 4 * cg), u1 = lds4(Us + (j + 1) * P + 4 * cg);
        const float4 u2 = lds4(Us + (j + 2) * P + 4 * cg), u3 = lds4(Us + (j + 3) * P + 4 * cg);
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
          const float4 m = lds4(Mq + (i0 + r) * MP + j);
          ao[r].x = fmaf(m.x, u0.x, fmaf(m.y, u1.x, fmaf(m.z, u2.x, fmaf(m.w, u3.x, ao[r].x))));
          ao[r].y = fmaf(m.x, u0.y, fmaf(m.y, u1.y, fmaf(m.z, u2.y, fmaf(m.w, u3.y, ao[r].y))));
          ao[r].z = fmaf(m.x, u0.z, fmaf(m.y, u1.z, fmaf(m.z, u2.z, fmaf(m.w, u3.z, ao[r].z))));
          ao[r].w = fmaf(m.x, u0.w, fmaf(m.y, u1.w, fmaf(m.z, u2.w, fmaf(m.w, u3.w, ao[r].w))));
        }
      }
#pragma unroll
      for (int r = 0; r < RPT; ++r) sts4(Qs + (i0 + r) * P + 4 * cg, ao[r]);

      constexpr int SPT = D / NRG;  // state rows per thread
      const int d0 = rg * SPT;
      const float gC = gam[C - 1];
      const float eC = expf(gC);
      float4 as[SPT];
#pragma unroll
      for (int r = 0; r < SPT; ++r) {
        const float4 sv = lds4(Ss + (d0 + r) * P + 4 * cg);
        as[r] = make_float4(eC * sv.x, eC * sv.y, eC * sv.z, eC * sv.w);
      }
#pragma unroll 1
      for (int i = 0; i < c; ++i) {
        const float w = expf(gC - gam[i]);
        const float4 u = lds4(Us + i * P + 4 * cg);
        const float4 uw = make_float4(w * u.x, w * u.y, w * u.z, w * u.w);
#pragma unroll
        for (int r4 = 0; r4 < SPT; r4 += 4) {
          const float4 kk = lds4(Ks + i * P + d0 + r4);
          const float kx[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            as[r4 + q].x = fmaf(kx[q], uw.x, as[r4 + q].x);
            as[r4 + q].y = fmaf(kx[q], uw.y, as[r4 + q].y);
            as[r4 + q].z = fmaf(kx[q], uw.z, as[r4 + q].z);
            as[r4 + q].w = fmaf(kx[q], uw.w, as[r4 + q].w);
          }
        }
      }
      __syncthreads();  // every thread is done reading S (K S above) before it is rewritten
#pragma unroll
      for (int r = 0; r < SPT; ++r) sts4(Ss + (d0 + r) * P + 4 * cg, as[r]);
    }
    __syncthreads();
    // ---- output rows: o rounded to T, then the fused gated RMSNorm (one warp per row); the z rows
    // are staged first in the K region (free now), all loads in flight at once
    const bool gated = a.z != nullptr;
    if (gated) {
      constexpr int EPV = 16 / (int)sizeof(T), VPR = D / EPV, NV = C * VPR / Y::kThreads;
      static_assert(C * VPR % Y::kThreads == 0, "z tiling");
      const T* zb = reinterpret_cast<const T*>(a.z) + (int64_t)vh * D;
      const bool zvec = ((reinterpret_cast<uintptr_t>(zb) | (uintptr_t)(a.z_stride_tok * (int64_t)sizeof(T))) & 15) == 0;
      if (zvec) {
        uint4 raw[NV];
#pragma unroll
        for (int n = 0; n < NV; ++n) {
          const int e = tid + n * Y::kThreads, i = e / VPR, vi = e - (e / VPR) * VPR;
          raw[n] = i < c ? *reinterpret_cast<const uint4*>(zb + (t0 + c0 + i) * a.z_stride_tok + vi * EPV)
                         : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int n = 0; n < NV; ++n) {
          const int e = tid + n * Y::kThreads, i = e / VPR, vi = e - (e / VPR) * VPR;
          const T* src = reinterpret_cast<const T*>(&raw[n]);
#pragma unroll
          for (int q = 0; q < EPV; ++q) Ks[i * P + vi * EPV + q] = to_f(src[q]);
        }
      } else {
#pragma unroll 4
        for (int e = tid; e < c * D; e += Y::kThreads) {
          const int i = e / D, d = e - (e / D) * D;
          Ks[i * P + d] = to_f(zb[(t0 + c0 + i) * a.z_stride_tok + d]);
        }
      }
      __syncthreads();
    }
    const T* wn = gated ? reinterpret_cast<const T*>(a.norm_weight) + (a.norm_weight_len == D ? 0 : (int64_t)vh * D)
                        : nullptr;
    for (int i = warp; i < c; i += Y::kThreads / 32) {
      const int64_t t = t0 + c0 + i;
      T* out = reinterpret_cast<T*>(a.out) + t * a.out_stride_tok + (int64_t)vh * D;
      float x[D / 32];
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < D / 32; ++k) {
        x[k] = round_to<T>(Qs[i * P + lane + 32 * k]);
        ss = fmaf(x[k], x[k], ss);
      }
      if (!gated) {
#pragma unroll
        for (int k = 0; k < D / 32; ++k) out[lane + 32 * k] = from_f<T>(x[k]);
        continue;
      }
      ss = warp_sum(ss);
      const float rs = rsqrtf(ss / (float)D + a.norm_eps);
#pragma unroll
      for (int k = 0; k < D / 32; ++k) {
        const int j = lane + 32 * k;
        out[j] = from_f<T>(to_f(wn[j]) * (x[k] * rs) * silu_f(Ks[i * P + j]));
      }
    }
    __syncthreads();  // the next chunk overwrites Q/K/U
  }
  for (int e = tid; e < D * NCG; e += Y::kThreads) {
    const int r = e / NCG, c4 = e - (e / NCG) * NCG;
    __stcs(reinterpret_cast<float4*>(st + (size_t)r * D) + c4, lds4(Ss + r * P + 4 * c4));
  }
}

template <int DK, int DV>
constexpr size_t decode_smem(int vpk) {
  return (size_t)(DK * DV + 2 * DK + 3 * vpk * DV + 16 * DV + 2 * DV + 4 + 2 * vpk) * 4;
}

template <typename T, int DK, int DV>
cudaError_t launch_decode_t(const tf_gdn_args& a, cudaStream_t s) {
  const int vpk = a.num_v_heads / a.num_k_heads;
  const size_t smem = decode_smem<DK, DV>(vpk);
  cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, DK, DV>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // persistent: as many CTAs as fit at once (2 per SM by the launch bounds, fewer when the
  // shared memory of a large vpk does not allow it), never more than there are items
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel<T, DK, DV>, 2 * DV, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  const int64_t items = (int64_t)a.batch_size * a.num_k_heads;
  const int64_t cap = (int64_t)device_sm_count() * per_sm;
  const int grid = (int)(items < cap ? items : cap);
  decode_kernel<T, DK, DV><<<grid, 2 * DV, smem, s>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// a7 on the 5th-generation tensor cores (dk = dv = 128, bf16 activations): the same chunked WY form,
// transposed so that the v dimension (128) is the MMA's M and lives on the TMEM lanes:
//   X   = [K; Q] K^T        (M128 N64: rows 0-63 K K^T, rows 64-127 Q K^T)
//   KS' = S' K^T,  QS' = S' Q^T     with S' = S^T [dv x dk] resident in TMEM across chunks
//   U'  = solve of (I + Mk) against beta (V - e^g KS)^T, one dv row per thread, in registers
//   O'  = e^g QS' + U' Mq^T,   S' = e^gC S' + U'' K      (U'' = U' o e^(gC - g))
// K and Q enter the products as the raw bf16 conv outputs: a product of two bf16 values is exact
// in the fp32 accumulator, so X takes one MMA per k-step, and the L2-norm factors 1/|k|, 1/|q| are
// applied to the products (in Mk, Mq, the solve's right side, O' and U'').  Products with an fp32
// operand (S', U', Mq) run as bf16 pairs x = hi + lo (hi = bf16(x), lo = bf16(x - hi)):
// S'.K = S'hi.K + S'lo.K, U'.Mq^T = hi.hi + hi.lo + lo.hi, about 2^-16 relative per product, which
// keeps the state within 1e-5 of the fp32 recurrence over thousands of tokens.  TMEM (512
// columns): S' fp32 128, S' hi/lo as bf16 pairs 64 + 64, X (then U'' hi/lo) 64, KS' 64, QS'/O' 64,
// U' hi/lo 32 + 32.
// Roles: warps 0-3 own TMEM lanes (solve, mask building, rescales, output with the fused gated
// RMSNorm), warps 4-7 copy the chunk's raw q/k rows into a SWIZZLE_128B [K; Q] stack and compute
// their norms and the per-token factors, v, silu(z) and the gates, warp 8 allocates TMEM and one
// of its threads issues the MMAs.
// ---------------------------------------------------------------------------------------------
namespace tc_chunk {

constexpr int C = 64, D = 128;
constexpr int kThreads = 288;
constexpr int kKQBlk = 128 * 128;             // one 64-dim block of a [K; Q] stack (128 rows)
constexpr int kStack = 2 * kKQBlk;            // a [K; Q] stack of raw bf16 rows, 32 KB
constexpr int kVBuf = C * D * 2;              // T [64][128] v rows
// Chunks alternate between two sets of the buffers the loaders fill (stack, v rows, per-token
// arrays), so that chunk c+1's rows are in place while chunk c still computes.
constexpr int oKQ = 0;                        // stacks [2]
constexpr int oV = 2 * kStack;                // v rows [2]
constexpr int oZ = oV + 2 * kVBuf;            // fp32 [64][128] silu(z) of the output gate
constexpr int oOT = oZ + C * D * 4;           // T [64][128] output rows (O' transposed, rounded)
constexpr int oMk = oOT + C * D * 2;          // fp32 [64 j][64 i]: Mk transposed
constexpr int oMqH = oMk + C * C * 4;         // bf16 [64 rows][128 B] K-major (SWIZZLE_128B)
constexpr int oMqL = oMqH + C * 128;
// The off-diagonal block Mk10 (rows 32-63, columns 0-31 of Mk) as the bf16 hi / lo B operand of
// the solve's tensor-core step: [32 rows][128 B] K-major (SWIZZLE_128B; K = 32, the first 64
// bytes of a row)
constexpr int kTile = 32 * 128;
constexpr int oM10H = oMqL + C * 128;
constexpr int oM10L = oM10H + kTile;
// per-token arrays [2][7][64]: gamma (log2 units), beta, 1/|k|, dk^-1/2/|q|, e^gamma/|k| (the
// solve's right side), e^gamma dk^-1/2/|q| (O' = e^g QS'), e^(gamma_C - gamma)/|k| (U'')
constexpr int oArr = oM10L + kTile;
constexpr int kArr = 7 * C * 4;
enum { aGam = 0, aBet, aInK, aInQ, aEk, aEq, aSk };
constexpr int oGr = oArr + 2 * kArr;          // raw g [64] (loaders)
constexpr int oBar = oGr + C * 4;             // in_full[2] p1 l1 p2[2] tm_free chunk_free fin rows_full[2] p1x sreq sdone p2s
constexpr int oWords = oBar + 128;            // tmem holder, abort
constexpr int oRawZ = (oWords + 16 + 1023) & ~1023;  // next chunk's raw z rows (T)
constexpr int kSmem = oRawZ + C * D * 2 + 1024;
static_assert(kSmem <= 232448, "shared memory per CTA");
constexpr int cS = 0, cSH = 128, cSL = 192, cX = 256, cY = 320, cZ = 384, cUH = 448, cUL = 480;
static_assert(oMqH % 1024 == 0 && oMqL % 1024 == 0 && kStack % 1024 == 0 && oM10H % 1024 == 0 &&
              kTile % 1024 == 0, "SWIZZLE_128B tiles are 1024-byte aligned");

// 2^x (ex2.approx.ftz: relative error about 2^-22)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;
// two fp32 values in one 64-bit register (x in the low half) and the paired fp32 FMA of sm_100
__device__ __forceinline__ uint64_t pack2(float x, float y) {
  return ((uint64_t)__float_as_uint(y) << 32) | __float_as_uint(x);
}
__device__ __forceinline__ float lo_of(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_of(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
// Warp reduce-scatter of N values per lane (N a power of two <= 32): halving exchanges at lane
// offsets 16, 8, ... leave lane L with the sum over the warp of value L >> (5 - log2 N), in
// N - 1 + (5 - log2 N) shuffles instead of 5 N; every lane of the value's group holds the total.
template <int N, int O>
__device__ __forceinline__ void rs_step(float* a, int lane) {
  if constexpr (O >= 1) {
    if constexpr (N > 1) {
      const bool up = (lane & O) != 0;
#pragma unroll
      for (int j = 0; j < N / 2; ++j) {
        const float keep = up ? a[j + N / 2] : a[j];
        const float send = up ? a[j] : a[j + N / 2];
        a[j] = keep + __shfl_xor_sync(0xffffffffu, send, O);
      }
      rs_step<N / 2, O / 2>(a, lane);
    } else {
      a[0] += __shfl_xor_sync(0xffffffffu, a[0], O);
      rs_step<1, O / 2>(a, lane);
    }
  }
}
template <int N>
__device__ __forceinline__ float reduce_scatter(const float (&v)[N], int lane) {
  float a[N];
#pragma unroll
  for (int j = 0; j < N; ++j) a[j] = v[j];
  rs_step<N, 16>(a, lane);
  return a[0];
}

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// x * sigmoid(x) with an approximate division (no slow path; 0 below x = -87, as the exact value is)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.and.pred q, %2, %3, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool waitb(uint64_t* bar, uint32_t parity, volatile int* abort) {
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
// x = hi + lo in bf16, packed as the pair (x0, x1) of one 32-bit column / word
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  __nv_bfloat162 l = __floats2bfloat162_rn(x0 - __low2float(h), x1 - __high2float(h));
  hi = *reinterpret_cast<uint32_t*>(&h);
  lo = *reinterpret_cast<uint32_t*>(&l);
}
__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void sts_v2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, bool acc) {
  tc::mma_bf16_ts(d, a, b, idesc, acc);
}
__device__ __forceinline__ void st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  float f[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(v[i]);
  tc::st16(taddr, f);
}

// four consecutive 16-bit elements of a staged row (8-byte aligned) as floats, or zeros
template <typename T>
__device__ __forceinline__ void load4(const T* p, bool live, float (&f)[4]) {
  static_assert(sizeof(T) == 2, "16-bit rows");
  uint2 u = live ? *reinterpret_cast<const uint2*>(p) : make_uint2(0u, 0u);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = to_f(e[j]);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) chunk_tc_kernel(tf_gdn_args a, const int64_t* start,
                                                               const T* conv_out, const int32_t* order,
                                                               const __grid_constant__ CUtensorMap map_qk,
                                                               const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023) & ~1023u;
  unsigned char* sb = smem_raw + (base - raw_base);
  float* MkT = reinterpret_cast<float*>(sb + oMk);
  float* graw = reinterpret_cast<float*>(sb + oGr);
  auto arr = [&](int buf, int k) { return reinterpret_cast<float*>(sb + oArr + buf * kArr + k * C * 4); };
  // A barrier used by chunks of one parity (in_full, p2) completes its phase for chunk c as its
  // (c >> 1)-th: no waiter can find it two phases ahead, since the next use needs this one's
  // consumers to have passed.
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + oBar);
  uint64_t* in_full = bars;            // [2] a chunk's stack, v rows and arrays are in place
  uint64_t* p1 = bars + 2;             // phase-1 products of the chunk are in TMEM
  uint64_t* l1 = bars + 3;             // Mq, U', U'' and the rescales are written
  uint64_t* p2 = bars + 4;             // [2] a chunk's phase-2 products have completed
  uint64_t* tm_free = bars + 6;        // S' hi / lo and the O' rows written: phase 1 may run
  uint64_t* chunk_free = bars + 7;     // the output rows are written: O' may replace them
  uint64_t* fin = bars + 8;            // every MMA of the CTA has completed
  uint64_t* rows_full = bars + 9;      // [2] a chunk's q, k, v rows have landed (TMA)
  uint64_t* p1x = bars + 11;           // X of the chunk is in TMEM (the rest of phase 1 follows)
  uint64_t* sreq = bars + 12;          // U'0 (the solved first 32 tokens) is in TMEM
  uint64_t* sdone = bars + 13;         // E = U'0 Mk10^T is in TMEM
  uint64_t* p2s = bars + 14;           // a chunk's state-update MMAs (S' += U'' K) have completed
                                       // (p2 of the chunk's parity: all its phase-2 MMAs)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sb + oWords);
  volatile int* abort = reinterpret_cast<volatile int*>(sb + oWords + 4);

  const int b = order[blockIdx.x / a.num_v_heads];
  const int vh = blockIdx.x % a.num_v_heads;
  const int kh = vh / (a.num_v_heads / a.num_k_heads);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int key_dim = a.num_k_heads * D;
  const int64_t slot = a.req_pool_indices[b];
  if (slot < 0 || slot >= a.num_slots) return;  // recorded by the conv kernel
  const int64_t t0 = start[b];
  const int64_t E = clamp_extend(a, b, t0);
  if (E <= 0) return;
  const int nchunks = (int)((E + C - 1) / C);
  float* st_g = a.ssm_state + slot * a.ssm_stride_slot + (size_t)vh * D * D;

  if (tid == 0) {
    mbar_init(in_full, 128);
    mbar_init(in_full + 1, 128);
    mbar_init(p1, 1);
    mbar_init(l1, 4);
    mbar_init(p2, 1);
    mbar_init(p2 + 1, 1);
    mbar_init(rows_full, 1);
    mbar_init(rows_full + 1, 1);
    mbar_init(p1x, 1);
    mbar_init(sreq, 4);
    mbar_init(sdone, 1);
    mbar_init(p2s, 1);
    mbar_init(tm_free, 4);
    mbar_init(chunk_free, 4);
    mbar_init(fin, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 8) tc::tmem_alloc(tmem_holder, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp >= 4 && warp < 8) {
    // ============ loaders: the chunk's raw q/k rows and norms, v, silu(z) and gates ============
    // The next chunk's raw rows are copied into a staging area with cp.async (every copy in
    // flight at once) while the current chunk computes; the copy into the MMA layouts starts as
    // soon as the lane warps release the working buffers.
    const int lt = tid - 128, lw = warp - 4;
    const float qscale = rsqrtf((float)D);
    const T* zb = a.z ? reinterpret_cast<const T*>(a.z) + (int64_t)vh * D : nullptr;
    const bool zvec = zb && ((reinterpret_cast<uintptr_t>(zb) | (uintptr_t)(a.z_stride_tok * 2)) & 15) == 0;
    // gates: the next chunk's raw a, b are loaded with its rows and turned into g, beta when the
    // chunk starts (the loads' latency overlaps this chunk), with the head's constants hoisted
    T a_next = from_f<T>(0.f), b_next = from_f<T>(0.f);
    bool gate_next = false;
    const float neg_ea = -expf(to_f(reinterpret_cast<const T*>(a.A_log)[vh]));
    const float dtb = to_f(reinterpret_cast<const T*>(a.dt_bias)[vh]);
    // A chunk's q, k, v rows arrive by TMA once chunk c-1's phase 2 has released the buffers of
    // its parity: six 64-row x 64-column boxes, q and k SWIZZLE_128B straight into the [K; Q]
    // stack (k rows 0-63, q rows 64-127 of each 64-dim block), v as two [64][64] halves; one
    // thread issues them.  Rows past the batch are zero-filled by the TMA unit, rows of the next
    // request are zeroed once they land.  The gates' raw a, b are loaded alongside; z is staged
    // raw by cp.async once the previous silu rows are written.
    int tma_pending = -1;  // the chunk whose rows were requested and not yet waited for
    auto prefetch_rows = [&](int ci) {
      const int64_t c0 = (int64_t)ci * C;
      const int c = (int)(E - c0 < C ? E - c0 : C);
      tma_pending = ci;
      if (lt == 0) {
        const uint32_t stk = base + oKQ + (ci & 1) * kStack, vbuf = base + oV + (ci & 1) * kVBuf;
        uint64_t* bar = rows_full + (ci & 1);
        const int row = (int)(t0 + c0);
        mbar_arrive_expect_tx(bar, 6 * C * 64 * 2);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tma::load_2d(stk + h * kKQBlk, &map_qk, key_dim + kh * D + 64 * h, row, bar);
          tma::load_2d(stk + h * kKQBlk + 64 * 128, &map_qk, kh * D + 64 * h, row, bar);
          tma::load_2d(vbuf + h * C * 128, &map_v, 2 * key_dim + vh * D + 64 * h, row, bar);
        }
      }
      if (lt < C) {
        gate_next = lt < c;
        if (gate_next) {
          const int64_t t = t0 + c0 + lt;
          a_next = reinterpret_cast<const T*>(a.a)[t * a.a_stride_tok + vh];
          b_next = reinterpret_cast<const T*>(a.b)[t * a.b_stride_tok + vh];
        }
      }
    };
    auto prefetch_z = [&](int ci) {
      const int64_t c0 = (int64_t)ci * C;
      const int c = (int)(E - c0 < C ? E - c0 : C);
#pragma unroll
      for (int n = 0; n < 8; ++n) {  // 64 rows x 16 pieces, 8 per loader thread
        const int e = lt + 128 * n;
        const int i = e >> 4, pc = e & 15;
        if (i < c) {
          const int64_t t = t0 + c0 + i;
          if (zvec) {
            cp_async16(base + oRawZ + (i * D + pc * 8) * 2, zb + t * a.z_stride_tok + pc * 8);
          } else if (zb) {
            T* dz = reinterpret_cast<T*>(sb + oRawZ + (i * D + pc * 8) * 2);
#pragma unroll
            for (int q = 0; q < 8; ++q) dz[q] = zb[t * a.z_stride_tok + pc * 8 + q];
          }
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const T* wn = a.z ? reinterpret_cast<const T*>(a.norm_weight) + (a.norm_weight_len == D ? 0 : (int64_t)vh * D)
                      : nullptr;
    float wv[4] = {0.f, 0.f, 0.f, 0.f};
    if (wn) {
#pragma unroll
      for (int e = 0; e < 4; ++e) wv[e] = to_f(wn[4 * lane + e]);
    }
    // output rows of chunk cj: o rounded to T (the lanes' O' rows), then the fused gated RMSNorm
    // with this warp's rows lw + 4m; the lanes may replace the O' rows once chunk_free completes
    auto out_rows = [&](int cj) -> bool {
      const int64_t c0 = (int64_t)cj * C;
      const int c = (int)(E - c0 < C ? E - c0 : C);
      if (!bar_and(2, 128, waitb(tm_free, (cj + 1) & 1, abort))) return false;
      const T* ot = reinterpret_cast<const T*>(sb + oOT);
      {
        const float* zs = reinterpret_cast<const float*>(sb + oZ);  // silu(z)
        T* outb = reinterpret_cast<T*>(a.out) + (t0 + c0) * a.out_stride_tok + (int64_t)vh * D + 4 * lane;
        const bool ovec = ((reinterpret_cast<uintptr_t>(a.out) | (uintptr_t)(a.out_stride_tok * 2)) & 7) == 0;
        // 8 rows at a time (rows lw + 4m): their squared norms reduce-scattered over the warp
#pragma unroll 1
        for (int bt = 0; bt < 2; ++bt) {
          if (lw + 32 * bt >= c) break;
          float x[8][4], part[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int i = lw + 4 * (8 * bt + j);
            load4(ot + i * D + 4 * lane, i < c, x[j]);
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) ss = fmaf(x[j][e], x[j][e], ss);
            part[j] = ss;
          }
          float rr = 1.f;
          if (wn) {
            const float tot = reduce_scatter<8>(part, lane);
            rr = rsqrtf(tot / (float)D + a.norm_eps);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int i = lw + 4 * (8 * bt + j);
            if (i >= c) break;
            float y[4];
            if (wn) {
              const float r = __shfl_sync(0xffffffffu, rr, 4 * j);
              const float4 zf = *reinterpret_cast<const float4*>(zs + i * D + 4 * lane);
              const float ze[4] = {zf.x, zf.y, zf.z, zf.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) y[e] = wv[e] * (x[j][e] * r) * ze[e];
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) y[e] = x[j][e];
            }
            T* out = outb + (int64_t)i * a.out_stride_tok;
            if (ovec) {
              *reinterpret_cast<uint2*>(out) =
                  make_uint2(pack2_rn<T>(y[0], y[1]), pack2_rn<T>(y[2], y[3]));
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) out[e] = from_f<T>(y[e]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(chunk_free);
      return true;
    };
    prefetch_rows(0);
    prefetch_z(0);
    bool ok = true;
    for (int ci = 0; ci < nchunks && ok; ++ci) {
      const int64_t c0 = (int64_t)ci * C;
      const int c = (int)(E - c0 < C ? E - c0 : C);
      const int bf = ci & 1;
      float* gam = arr(bf, aGam);
      float* bet = arr(bf, aBet);
      float* ink = arr(bf, aInK);
      float* inq = arr(bf, aInQ);
      float* ekf = arr(bf, aEk);
      float* eqf = arr(bf, aEq);
      float* skf = arr(bf, aSk);
      ok = bar_and(2, 128, waitb(rows_full + bf, (ci >> 1) & 1, abort));  // q, k, v have landed
      if (!ok) break;
      tma_pending = -1;
      if (c < C) {  // rows past the request's end (the next request's, or zero fill) become zeros
        const uint32_t stk = oKQ + bf * kStack, vbuf = oV + bf * kVBuf;
        for (int e = lt; e < (C - c) * 48; e += 128) {  // 48 pieces of 16 bytes per row
          const int i = c + e / 48, pc = e % 48;
          uint32_t off;
          if (pc < 32) {  // k (pc < 16) or q row, 128-byte swizzled block rows: zero as a whole
            const int r = pc < 16 ? i : 64 + i;
            off = stk + ((pc >> 3) & 1) * kKQBlk + r * 128 + (pc & 7) * 16;
          } else {
            off = vbuf + ((pc >> 3) & 1) * C * 128 + i * 128 + (pc & 7) * 16;
          }
          *reinterpret_cast<uint4*>(sb + off) = make_uint4(0u, 0u, 0u, 0u);
        }
        named_barrier(2, 128);
      }
      if (lt < C) {
        // g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)  (linear_attention.py:178-181)
        graw[lt] = gate_next ? neg_ea * softplus_f(to_f(a_next) + dtb) : 0.f;
        bet[lt] = gate_next ? 1.0f / (1.0f + expf(-to_f(b_next))) : 0.f;
      }
      const T* rz = reinterpret_cast<const T*>(sb + oRawZ);
      const uint32_t stk = base + oKQ + bf * kStack;
      const int d = 4 * lane;               // this lane's 4 elements of a row
      const int blk = lane >> 4, ch = (lane & 15) >> 1, e8 = (lane & 1) * 4;
      // the norms of the rows in the stack, 8 rows at a time: the 16 squared norms (8 q, 8 k)
      // reduce-scattered over the warp, one rsqrt per lane.  The raw rows are the MMA operands:
      // bf16 products are exact in the fp32 accumulators, and the 1/|q|, 1/|k| factors are
      // applied to the products
#pragma unroll 1
      for (int bt = 0; bt < 2; ++bt) {
        float part[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = lw + 4 * (8 * bt + j);
          const int rk_ = i, rq_ = 64 + i;
          const uint32_t ok_ = (uint32_t)blk * kKQBlk + ((uint32_t)(ch ^ (rk_ & 7)) << 4) + e8 * 2;
          const uint32_t oq_ = (uint32_t)blk * kKQBlk + ((uint32_t)(ch ^ (rq_ & 7)) << 4) + e8 * 2;
          const uint2 kr = *reinterpret_cast<const uint2*>(sb + (stk - base) + rk_ * 128 + ok_);
          const uint2 qr = *reinterpret_cast<const uint2*>(sb + (stk - base) + rq_ * 128 + oq_);
          const float q0 = unpack_lo<T>(qr.x), q1 = unpack_hi<T>(qr.x), q2 = unpack_lo<T>(qr.y),
                      q3 = unpack_hi<T>(qr.y);
          const float k0 = unpack_lo<T>(kr.x), k1 = unpack_hi<T>(kr.x), k2 = unpack_lo<T>(kr.y),
                      k3 = unpack_hi<T>(kr.y);
          part[j] = fmaf(q3, q3, fmaf(q2, q2, fmaf(q1, q1, q0 * q0)));
          part[8 + j] = fmaf(k3, k3, fmaf(k2, k2, fmaf(k1, k1, k0 * k0)));
        }
        // x / max(|x|, 1e-12) as x * rsqrt(max(|x|^2, 1e-24)): no division on this path.  Lane
        // 2j holds q row j's factor, lane 16 + 2j k row j's
        const float tot = reduce_scatter<16>(part, lane);
        const float rn = ((lane >> 1) < 8 ? qscale : 1.f) * rsqrtf(fmaxf(tot, 1e-24f));
        if ((lane & 1) == 0) (lane < 16 ? inq : ink)[lw + 4 * (8 * bt + ((lane >> 1) & 7))] = rn;
      }
      named_barrier(2, 128);  // graw complete
      if (lw == 0) {  // gamma = inclusive cumulative sum of g over the chunk, in log2 units
        const float g0 = graw[2 * lane] * kLog2e, g1 = graw[2 * lane + 1] * kLog2e;
        float incl = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        gam[2 * lane] = incl - g1;
        gam[2 * lane + 1] = incl;
        // the per-token factors of the products (every loader's norms are in place)
        const float gC = __shfl_sync(0xffffffffu, incl, 31);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * lane + h;
          const float gi = h ? incl : incl - g1, eg = ex2(gi);
          ekf[i] = eg * ink[i];
          eqf[i] = eg * inq[i];
          skf[i] = ex2(gC - gi) * ink[i];
        }
      }
      tc::fence_proxy_async_smem();  // the [K; Q] stack is read by the tensor core
      mbar_arrive(in_full + bf);
      // the next chunk's rows, into the buffers chunk ci-1 used, once its phase 2 has completed
      if (ci + 1 < nchunks) {
        if (!bar_and(2, 128, ci == 0 || waitb(p2 + (bf ^ 1), ((ci - 1) >> 1) & 1, abort))) {
          ok = false;
          break;
        }
        prefetch_rows(ci + 1);
      }
      // the previous chunk's output rows (its silu(z) rows are still in oZ), then this chunk's
      // silu(z): the gate's exponentials and divisions and the output rows run here, beside the
      // lanes' work on this chunk, instead of on the lanes' critical path
      if (ci > 0 && !out_rows(ci - 1)) { ok = false; break; }
      asm volatile("cp.async.wait_group 0;" ::: "memory");  // this chunk's z
      ok = bar_and(2, 128, ok);
      if (!ok) break;
#pragma unroll 4
      for (int m = 0; m < 16; ++m) {
        const int i = lw + 4 * m;
        float z[4];
        load4(rz + i * D + d, i < c && zb, z);
        sts_v4(base + oZ + (i * D + d) * 4, __float_as_uint(silu_fast(z[0])),
               __float_as_uint(silu_fast(z[1])), __float_as_uint(silu_fast(z[2])),
               __float_as_uint(silu_fast(z[3])));
      }
      named_barrier(2, 128);  // the z staging is consumed before it is refilled
      if (ci + 1 < nchunks) prefetch_z(ci + 1);
    }
    if (ok) out_rows(nchunks - 1);
    asm volatile("cp.async.wait_all;" ::: "memory");
    // after an abort, rows still in flight land before the CTA (and its shared memory) ends
    if (lt == 0 && tma_pending >= 0) mbar_wait(rows_full + (tma_pending & 1), (tma_pending >> 1) & 1);
  } else if (warp == 8) {
    // ============ MMA issue (one thread) ============
    if (lane == 0) {
      constexpr uint32_t idX = tc::idesc_bf16(128, 64, false, false);
      constexpr uint32_t idYZ = tc::idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = tc::idesc_bf16(128, 64, false, false);
      constexpr uint32_t idS = tc::idesc_bf16(128, 128, false, true);
      constexpr uint32_t idB = tc::idesc_bf16(128, 32, false, false);
      for (int ci = 0; ci < nchunks; ++ci) {
        const int bf = ci & 1;
        const uint32_t kq = base + oKQ + bf * kStack;
        if (!waitb(tm_free, ci & 1, abort) || !waitb(in_full + bf, (ci >> 1) & 1, abort)) break;
        tc::fence_proxy_async_smem();
        tc::fence_after_sync();
        // X = [K; Q] K^T of the raw rows (exact bf16 products: one MMA per k-step), committed on
        // its own so that the masks start early; then KS' = S' K^T and QS' = S' Q^T as
        // S'hi.K + S'lo.K
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t bKQ = tc::sw128_desc(kq + (kk >> 2) * kKQBlk + (kk & 3) * 32, 16, 1024);
          tc::mma_bf16(tmem + cX, bKQ, bKQ, idX, kk > 0);
        }
        tc::commit(p1x);
#pragma unroll 1
        for (int part = 0; part < 2; ++part) {
          const uint32_t aT = tmem + (part ? cSL : cSH);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kKQBlk + (kk & 3) * 32;
            const uint64_t bKQ = tc::sw128_desc(kq + off, 16, 1024);  // K rows, then Q rows
            mma_ts(tmem + cY, aT + kk * 8, bKQ, idYZ, part > 0 || kk > 0);  // [KS' | QS'] over cY, cZ
          }
        }
        tc::commit(p1);
        if (!waitb(sreq, ci & 1, abort)) break;
        tc::fence_after_sync();
        tc::fence_proxy_async_smem();
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          mma_ts(tmem + cX + 32, tmem + cUH + kk * 8, tc::sw128_desc(base + oM10H + kk * 32, 16, 1024), idB, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          mma_ts(tmem + cX + 32, tmem + cUH + kk * 8, tc::sw128_desc(base + oM10L + kk * 32, 16, 1024), idB, true);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          mma_ts(tmem + cX + 32, tmem + cUL + kk * 8, tc::sw128_desc(base + oM10H + kk * 32, 16, 1024), idB, true);
        tc::commit(sdone);
        if (!waitb(l1, ci & 1, abort)) break;
        tc::fence_after_sync();
        tc::fence_proxy_async_smem();
        // O' += U' Mq^T (N = 64 tokens, hi.hi + hi.lo + lo.hi) and S' += U'' K (N = 128 dk, the
        // raw K rows MN-major; U'' = U' e^(gamma_C - gamma) / |k| as hi + lo over cX)
        // the state update first, committed on its own (p2s): the lanes split S' while the output
        // products run; p2 then completes once every phase-2 product has
#pragma unroll 1
        for (int part = 0; part < 2; ++part) {
          const uint32_t aK = tmem + cX + (part ? 32 : 0);
#pragma unroll
          for (int kk = 0; kk < C / 16; ++kk)
            mma_ts(tmem + cS, aK + kk * 8, tc::sw128_desc(kq + kk * 2048, kKQBlk, 1024), idS, true);
        }
        tc::commit(p2s);
#pragma unroll 1
        for (int part = 0; part < 3; ++part) {
          const uint32_t aT = tmem + (part == 2 ? cUL : cUH);
          const uint32_t mq = base + (part == 1 ? oMqL : oMqH);
#pragma unroll
          for (int kk = 0; kk < C / 16; ++kk)
            mma_ts(tmem + cZ, aT + kk * 8, tc::sw128_desc(mq + kk * 32, 16, 1024), idO, true);
        }
        tc::commit(p2 + bf);
      }
      // every MMA issued has completed before TMEM is read for the last time or released; the
      // issuing thread also waits for it (bounded), so that after an abort no MMA is in flight
      // when TMEM is released
      tc::commit(fin);
      mbar_wait(fin, 0);
    }
    __syncwarp();
  } else {
    // ============ TMEM-lane warps: thread l owns dv row l of S', KS', O', U' ============
    const int l = tid;
    const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
    bool ok = true;
    {  // S' = S^T into TMEM, with its bf16 hi / lo split; 64 loads in flight per thread
#pragma unroll 1
      for (int c2 = 0; c2 < 2; ++c2) {
        float sv[64];
#pragma unroll
        for (int k = 0; k < 64; ++k) sv[k] = __ldcs(st_g + (size_t)(c2 * 64 + k) * D + l);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int cc = 2 * c2 + h;
          tc::st32(lb + cS + cc * 32, *reinterpret_cast<float(*)[32]>(&sv[32 * h]));
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) split2(sv[32 * h + 2 * k], sv[32 * h + 2 * k + 1], hi[k], lo[k]);
          st16u(lb + cSH + cc * 16, hi);
          st16u(lb + cSL + cc * 16, lo);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(tm_free);
        mbar_arrive(chunk_free);
      }
    }
    for (int ci = 0; ci < nchunks; ++ci) {
      const int bf = ci & 1;
      const float* gam = arr(bf, aGam);
      const float* bet = arr(bf, aBet);
      const float* ink = arr(bf, aInK);
      const float* inq = arr(bf, aInQ);
      const float* ekf = arr(bf, aEk);
      const float* eqf = arr(bf, aEq);
      const float* skf = arr(bf, aSk);
      ok = bar_and(1, 128, ok && waitb(in_full + bf, (ci >> 1) & 1, abort) && waitb(p1x, ci & 1, abort));
      if (!ok) break;
      tc::fence_after_sync();
      // ---- rows of X: Mk (l < 64, stored transposed) or Mq (l >= 64, bf16 hi / lo K-major rows)
      {
        float x[64];
        tc::ld32(lb + cX, *reinterpret_cast<float(*)[32]>(&x[0]));
        tc::ld32(lb + cX + 32, *reinterpret_cast<float(*)[32]>(&x[32]));
        tc::wait_ld();
        const int i = l & 63;
        const float gi = gam[i];
        const float4* g4 = reinterpret_cast<const float4*>(gam);
        const float4* n4 = reinterpret_cast<const float4*>(ink);
        if (l < 64) {  // Mk_ij = beta_i e^(g_i - g_j) k_i.k_j / (|k_i| |k_j|), strictly lower
          // stored transposed for the register solves; rows 32-63 (warp 1) also write their
          // columns 0-31, the block Mk10, as the bf16 hi / lo B operand of the tensor-core step
          const float bi = bet[i] * ink[i];
#pragma unroll
          for (int j4 = 0; j4 < 16; ++j4) {
            const float4 g = g4[j4], n = n4[j4];
            const float gj[4] = {g.x, g.y, g.z, g.w}, nj[4] = {n.x, n.y, n.z, n.w};
            float m[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 4 * j4 + e;
              m[e] = j < i ? bi * ex2(gi - gj[e]) * (x[j] * nj[e]) : 0.f;
              MkT[j * C + i] = m[e];
            }
            if (j4 < 8 && l >= 32) {
              uint32_t h0, h1, l0, l1_;
              split2(m[0], m[1], h0, l0);
              split2(m[2], m[3], h1, l1_);
              const int ib = i - 32;
              const uint32_t off = ib * 128 + ((uint32_t)((j4 >> 1) ^ (ib & 7)) << 4) + (j4 & 1) * 8;
              sts_v2(base + oM10H + off, h0, h1);
              sts_v2(base + oM10L + off, l0, l1_);
            }
          }
        } else {  // Mq_ij = e^(g_i - g_j) q_i.k_j dk^-1/2 / (|q_i| |k_j|)
          const float qi = inq[i];
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const float4 ga = g4[2 * c8], gb = g4[2 * c8 + 1];
            const float4 na = n4[2 * c8], nb = n4[2 * c8 + 1];
            const float gj[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
            const float nj[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
            uint32_t h[4], lo_[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j0 = 8 * c8 + 2 * e, j1 = j0 + 1;
              const float m0 = j0 <= i ? qi * ex2(gi - gj[2 * e]) * (x[j0] * nj[2 * e]) : 0.f;
              const float m1 = j1 <= i ? qi * ex2(gi - gj[2 * e + 1]) * (x[j1] * nj[2 * e + 1]) : 0.f;
              split2(m0, m1, h[e], lo_[e]);
            }
            const uint32_t off = i * 128 + ((uint32_t)(c8 ^ (i & 7)) << 4);
            sts_v4(base + oMqH + off, h[0], h[1], h[2], h[3]);
            sts_v4(base + oMqL + off, lo_[0], lo_[1], lo_[2], lo_[3]);
          }
        }
      }
      ok = bar_and(1, 128, waitb(p1, ci & 1, abort));  // KS', QS' (and the masks are written)
      if (!ok) break;
      tc::fence_after_sync();
      // ---- U' row l: (I + Mk) U' = U with U = beta (v - e^g KS), in two halves of 32 tokens:
      //      tokens 0-31 solved in registers, their terms on tokens 32-63 (E = U'0 Mk10^T, half
      //      of the solve's products) on the tensor core, then tokens 32-63 in registers.  The
      //      register solves are right-looking: once u_j is final, every later row of the half
      //      takes its term (independent FMAs; column j of Mk is contiguous), rows (2p, 2p+1)
      //      packed in one 64-bit register and updated by one fma.rn.f32x2
      {
        uint64_t u2[32];
        {
          float u[64];
          tc::ld32(lb + cY, *reinterpret_cast<float(*)[32]>(&u[0]));
          tc::ld32(lb + cY + 32, *reinterpret_cast<float(*)[32]>(&u[32]));
          tc::wait_ld();
          // v rows as two [64][64] halves: element (i, l) at (l / 64) * 4096 + i * 64 + l % 64
          const T* vr = reinterpret_cast<const T*>(sb + oV + bf * kVBuf) + (l >> 6) * (C * 64) + (l & 63);
#pragma unroll
          for (int i = 0; i < 64; ++i) u[i] = bet[i] * (to_f(vr[i * 64]) - ekf[i] * u[i]);
#pragma unroll
          for (int p = 0; p < 32; ++p) u2[p] = pack2(u[2 * p], u[2 * p + 1]);
        }
#pragma unroll
        for (int j = 0; j < 31; ++j) {
          const float uj = (j & 1) ? hi_of(u2[j >> 1]) : lo_of(u2[j >> 1]);
          const uint64_t nuj = pack2(-uj, -uj);
#pragma unroll
          for (int q4 = (j + 1) >> 2; q4 < 8; ++q4) {
            const ulonglong2 m = *reinterpret_cast<const ulonglong2*>(MkT + j * C + 4 * q4);
            if (4 * q4 + 1 > j) u2[2 * q4] = ffma2(m.x, nuj, u2[2 * q4]);
            u2[2 * q4 + 1] = ffma2(m.y, nuj, u2[2 * q4 + 1]);
          }
        }
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) split2(lo_of(u2[k]), hi_of(u2[k]), hi[k], lo[k]);
        st16u(lb + cUH, hi);
        st16u(lb + cUL, lo);
        tc::wait_st();
        tc::fence_before_sync();
        tc::fence_proxy_async_smem();  // Mk10 is read by the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(sreq);
        ok = bar_and(1, 128, waitb(sdone, ci & 1, abort));
        if (!ok) break;
        tc::fence_after_sync();
        {
          float e[32];
          tc::ld32(lb + cX + 32, e);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 16; ++k) u2[16 + k] = pack2(lo_of(u2[16 + k]) - e[2 * k], hi_of(u2[16 + k]) - e[2 * k + 1]);
        }
#pragma unroll
        for (int j = 32; j < 63; ++j) {
          const float uj = (j & 1) ? hi_of(u2[j >> 1]) : lo_of(u2[j >> 1]);
          const uint64_t nuj = pack2(-uj, -uj);
#pragma unroll
          for (int q4 = (j + 1) >> 2; q4 < 16; ++q4) {
            const ulonglong2 m = *reinterpret_cast<const ulonglong2*>(MkT + j * C + 4 * q4);
            if (4 * q4 + 1 > j) u2[2 * q4] = ffma2(m.x, nuj, u2[2 * q4]);
            u2[2 * q4 + 1] = ffma2(m.y, nuj, u2[2 * q4 + 1]);
          }
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) split2(lo_of(u2[16 + k]), hi_of(u2[16 + k]), hi[k], lo[k]);
        st16u(lb + cUH + 16, hi);
        st16u(lb + cUL + 16, lo);
        // U'' = U' e^(gamma_C - gamma) / |k| (the state update's A) over cX
        const float2* s2 = reinterpret_cast<const float2*>(skf);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float2 sf = s2[16 * h + k];
            split2(lo_of(u2[16 * h + k]) * sf.x, hi_of(u2[16 * h + k]) * sf.y, hi[k], lo[k]);
          }
          st16u(lb + cX + 16 * h, hi);
          st16u(lb + cX + 32 + 16 * h, lo);
        }
      }
      // ---- O' = e^g QS' (the MMA adds U' Mq^T), S' *= e^gC
      {
        float zq[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tc::ld32(lb + cZ + 32 * h, zq);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) zq[k] *= eqf[32 * h + k];
          tc::st32(lb + cZ + 32 * h, zq);
        }
        const float gC = gam[C - 1], eC = ex2(gC);
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          tc::ld32(lb + cS + 32 * cc, zq);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) zq[k] *= eC;
          tc::st32(lb + cS + 32 * cc, zq);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      tc::fence_proxy_async_smem();  // Mq is read by the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(l1);
      // ---- S' hi / lo for the next chunk once the state update has completed (the output
      //      products may still run), then O' rounded to T into the transposed output rows; then
      //      the next chunk's products start while the loaders write the output rows
      ok = bar_and(1, 128, waitb(p2s, ci & 1, abort));
      if (!ok) break;
      tc::fence_after_sync();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float sv[32];
        tc::ld32(lb + cS + 32 * cc, sv);
        tc::wait_ld();
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) split2(sv[2 * k], sv[2 * k + 1], hi[k], lo[k]);
        st16u(lb + cSH + 16 * cc, hi);
        st16u(lb + cSL + 16 * cc, lo);
      }
      // the previous chunk's output rows are written by the loaders before O' replaces them
      ok = bar_and(1, 128, waitb(p2 + bf, (ci >> 1) & 1, abort) && waitb(chunk_free, ci & 1, abort));
      if (!ok) break;
      tc::fence_after_sync();
      T* ot = reinterpret_cast<T*>(sb + oOT);
      {
        float o[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tc::ld32(lb + cZ + 32 * h, o);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) ot[(32 * h + k) * D + l] = from_f<T>(o[k]);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(tm_free);
    }
    if (ok) {  // the state back to the pool
      ok = waitb(fin, 0, abort);
      tc::fence_after_sync();
#pragma unroll 1
      for (int cc = 0; cc < 4 && ok; ++cc) {
        float sv[32];
        tc::ld32(lb + cS + 32 * cc, sv);
        tc::wait_ld();
#pragma unroll
        for (int k = 0; k < 32; ++k) __stcs(st_g + (size_t)(cc * 32 + k) * D + l, sv[k]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && *abort) record_err(a.err, TF_KERR_TIMEOUT);
  tc::fence_after_sync();
  if (warp == 8) tc::tmem_dealloc(tmem, 512);
}

}  // namespace tc_chunk

struct ExtWs {
  int64_t* start;  // [B+1]
  int32_t* order;  // [B] requests by decreasing extend length
  void* conv_out;  // [T, conv_dim] of T
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

inline ExtWs carve_ext(void* base, const tf_gdn_args& a) {
  ExtWs w;
  w.start = (int64_t*)base;
  const size_t o1 = align256((size_t)(a.batch_size + 1) * 8);
  w.order = (int32_t*)((char*)base + o1);
  w.conv_out = (char*)base + o1 + align256((size_t)a.batch_size * 4);
  return w;
}

template <typename T, int DK, int DV>
cudaError_t launch_extend_t(const tf_gdn_args& a, void* ws, cudaStream_t s) {
  ExtWs w = carve_ext(ws, a);
  const int conv_dim = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
  offsets_kernel<<<1, 32, 0, s>>>(a.extend_lens, a.batch_size, w.start);
  order_kernel<<<1, 256, 0, s>>>(a.extend_lens, a.batch_size, w.order);
  const bool conv_vec = sizeof(T) == 2 && a.conv_kernel == 4 && conv_dim % 4 == 0 &&
                        a.qkv_stride_tok % 4 == 0 && (reinterpret_cast<uintptr_t>(a.qkv) & 7) == 0;
  if (conv_vec) {
    if constexpr (sizeof(T) == 2) {
      constexpr int kSpan = kConvVecTok * kConvPipeBlocks;
      dim3 cg((conv_dim / 4 + kConvVecThreads - 1) / kConvVecThreads,
              (unsigned)((a.num_tokens + kSpan - 1) / kSpan));
      conv4_pipe_kernel<T><<<cg, kConvVecThreads, 0, s>>>(a, w.start, (T*)w.conv_out);
    }
  } else if (a.conv_kernel == 4 && conv_dim % 2 == 0) {
    dim3 cg((conv_dim / 2 + kConvThreads - 1) / kConvThreads,
            (unsigned)((a.num_tokens + kConvTok - 1) / kConvTok));
    conv4_tiled_kernel<T><<<cg, kConvThreads, 0, s>>>(a, w.start, (T*)w.conv_out);
  } else {
    conv_extend_kernel<T><<<a.num_tokens, 256, 0, s>>>(a, w.start, (T*)w.conv_out);
  }
  dim3 rg((conv_dim + 255) / 256, a.batch_size);
  conv_state_roll_kernel<T><<<rg, 256, 0, s>>>(a, w.start);
  if constexpr (std::is_same<T, __nv_bfloat16>::value && DK == 128 && DV == 128) {  // tcgen05
    const size_t tsmem = tc_chunk::kSmem;
    cudaError_t e = cudaFuncSetAttribute(tc_chunk::chunk_tc_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem);
    if (e != cudaSuccess) return e;
    // the conv outputs [T, conv_dim] in 64 x 64 boxes: q, k SWIZZLE_128B (the MMA layout), v plain
    CUtensorMap map_qk, map_v;
    const uint64_t stride = (uint64_t)conv_dim * sizeof(T);
    if (!tma::map_2d_u16(&map_qk, w.conv_out, (uint64_t)a.num_tokens, (uint64_t)conv_dim, stride,
                         64, tc_chunk::C, true) ||
        !tma::map_2d_u16(&map_v, w.conv_out, (uint64_t)a.num_tokens, (uint64_t)conv_dim, stride,
                         64, tc_chunk::C, false))
      return cudaErrorInvalidValue;
    tc_chunk::chunk_tc_kernel<T><<<a.batch_size * a.num_v_heads, tc_chunk::kThreads, tsmem, s>>>(
        a, w.start, (const T*)w.conv_out, w.order, map_qk, map_v);
    return cudaGetLastError();
  }
  if constexpr (DK == DV && (DK == 64 || DK == 128)) {  // a7: chunked form
    constexpr size_t csmem = ChunkLay<DK>::kBytes;
    cudaError_t e = cudaFuncSetAttribute(chunk_extend_kernel<T, DK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem);
    if (e != cudaSuccess) return e;
    chunk_extend_kernel<T, DK><<<a.batch_size * a.num_v_heads, ChunkLay<DK>::kThreads, csmem, s>>>(
        a, w.start, (const T*)w.conv_out);
    return cudaGetLastError();
  }
  const size_t smem = (size_t)(2 * DK + DV + 16 * DV + 2 * DV + 4 + 2) * 4;
  cudaError_t e = cudaFuncSetAttribute(recurrent_extend_kernel<T, DK, DV>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  recurrent_extend_kernel<T, DK, DV><<<a.batch_size * a.num_v_heads, 2 * DV, smem, s>>>(
      a, w.start, (const T*)w.conv_out);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_decode(const tf_gdn_args& a, cudaStream_t s) {
  const int dk = a.head_k_dim, dv = a.head_v_dim;
  if (dk == 128 && dv == 128) return launch_decode_t<T, 128, 128>(a, s);
  if (dk == 64 && dv == 64) return launch_decode_t<T, 64, 64>(a, s);
  if (dk == 32 && dv == 32) return launch_decode_t<T, 32, 32>(a, s);
  if (dk == 16 && dv == 16) return launch_decode_t<T, 16, 16>(a, s);
  return cudaErrorNotSupported;
}

template <typename T>
cudaError_t dispatch_extend(const tf_gdn_args& a, void* ws, cudaStream_t s) {
  const int dk = a.head_k_dim, dv = a.head_v_dim;
  if (dk == 128 && dv == 128) return launch_extend_t<T, 128, 128>(a, ws, s);
  if (dk == 64 && dv == 64) return launch_extend_t<T, 64, 64>(a, ws, s);
  if (dk == 32 && dv == 32) return launch_extend_t<T, 32, 32>(a, ws, s);
  if (dk == 16 && dv == 16) return launch_extend_t<T, 16, 16>(a, ws, s);
  return cudaErrorNotSupported;
}

}  // namespace gdn

bool gdn_dims_supported(int dk, int dv) {
  return dk == dv && (dk == 16 || dk == 32 || dk == 64 || dk == 128);
}

cudaError_t launch_gdn_decode(const tf_gdn_args& a, cudaStream_t s) {
  if (a.batch_size == 0) return cudaSuccess;
  switch (a.dtype) {
    case TF_DTYPE_F32: return gdn::dispatch_decode<float>(a, s);
    case TF_DTYPE_BF16: return gdn::dispatch_decode<__nv_bfloat16>(a, s);
    default: return gdn::dispatch_decode<__half>(a, s);
  }
}

size_t gdn_extend_workspace(const tf_gdn_args& a) {
  const int conv_dim = 2 * a.num_k_heads * a.head_k_dim + a.num_v_heads * a.head_v_dim;
  const size_t eb = a.dtype == TF_DTYPE_F32 ? 4 : 2;
  return gdn::align256((size_t)(a.batch_size + 1) * 8) + gdn::align256((size_t)a.batch_size * 4) +
         (size_t)a.num_tokens * conv_dim * eb;
}

cudaError_t launch_gdn_extend(const tf_gdn_args& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  (void)ws_bytes;
  if (a.batch_size == 0 || a.num_tokens == 0) return cudaSuccess;
  switch (a.dtype) {
    case TF_DTYPE_F32: return gdn::dispatch_extend<float>(a, ws, s);
    case TF_DTYPE_BF16: return gdn::dispatch_extend<__nv_bfloat16>(a, ws, s);
    default: return gdn::dispatch_extend<__half>(a, ws, s);
  }
}

}  // namespace tf
