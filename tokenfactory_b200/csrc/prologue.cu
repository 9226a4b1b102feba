// Fused full-attention prologue (qwen3_8/full_attention.py:142-149): q/k RMSNorm
// (qwen3_8/rms_norm.py:19-24), partial (M-)RoPE (qwen3_8/rotary_embedding.py:46-95) and the KV-pool
// store, one read of q/k/v and one write of q_out and the pool rows.  HBM-bound.
//
// One CTA per token: its threads first compute the token's cos/sin (rounded to the dtype, as the
// reference casts them) into shared memory, then each warp takes whole rows — the Hq q-heads, the
// Hkv k-heads (both normalised and rotated) and the Hkv v-heads (copied).  Lane l holds elements
// d = l + 32 i of a row, so loads and stores are coalesced whatever the strides, and the rotation
// partner d +- rotary_dim/2 is in the same lane (half a multiple of 32) or in lane l ^ half
// (half a power of two below 32).
#include "common.cuh"
#include "launch.h"

namespace tf {
namespace prologue {

constexpr int kThreads = 256;
constexpr int kMaxD = 256;
constexpr int kTPC = 4;  // tokens per CTA of the vector form

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) prologue_kernel(tf_attn_prologue_args a) {
  constexpr int E = D / 32;  // elements per lane
  __shared__ float cs[kMaxD / 2], sn[kMaxD / 2];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = a.rotary_dim / 2;
  for (int j = tid; j < half; j += kThreads) {
    int row = 0;
    if (a.pos_rows == 3) {
      if (a.mrope_interleaved) {
        const int m = j % 3;
        if (m == 1 && j < 3 * a.mrope_section[1]) row = 1;
        else if (m == 2 && j < 3 * a.mrope_section[2]) row = 2;
      } else {
        row = j < a.mrope_section[0] ? 0 : (j < a.mrope_section[0] + a.mrope_section[1] ? 1 : 2);
      }
    }
    const float f = (float)a.positions[row * a.pos_stride + t] * a.inv_freq[j];
    cs[j] = round_to<T>(cosf(f));
    sn[j] = round_to<T>(sinf(f));
  }
  __syncthreads();

  int64_t loc = a.out_cache_loc[t];
  if (loc < 0) loc += a.num_slots;  // torch index semantics
  const bool loc_ok = loc >= 0 && loc < a.num_slots;
  if (!loc_ok && tid == 0) record_err(a.err, TF_KERR_SLOT_RANGE);

  const int Hq = a.num_q_heads, Hkv = a.num_kv_heads;
  const int nrows = Hq + 2 * Hkv;
  const bool wf32 = a.norm_weight_dtype == TF_DTYPE_F32;
  for (int r = warp; r < nrows; r += kThreads / 32) {
    const T* src;
    T* dst;
    if (r < Hq) {
      src = reinterpret_cast<const T*>(a.q) + t * a.q_stride_tok + (int64_t)r * a.q_stride_head;
      dst = reinterpret_cast<T*>(a.q_out) + t * a.q_out_stride_tok + (int64_t)r * a.q_out_stride_head;
    } else {
      if (!loc_ok) continue;
      const int h = r < Hq + Hkv ? r - Hq : r - Hq - Hkv;
      const bool isk = r < Hq + Hkv;
      src = reinterpret_cast<const T*>(isk ? a.k : a.v) + t * (isk ? a.k_stride_tok : a.v_stride_tok) +
            (int64_t)h * (isk ? a.k_stride_head : a.v_stride_head);
      dst = reinterpret_cast<T*>(isk ? a.k_buffer : a.v_buffer) + loc * a.buf_stride_slot +
            (int64_t)h * a.buf_stride_head;
    }
    float x[E];
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = to_f(src[lane + 32 * i]);
    if (r >= Hq + Hkv) {  // v: copied as is
#pragma unroll
      for (int i = 0; i < E; ++i) dst[lane + 32 * i] = from_f<T>(x[i]);
      continue;
    }
    const void* w = r < Hq ? a.q_norm_weight : a.k_norm_weight;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + a.eps);
    float y[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int d = lane + 32 * i;
      const float wv = wf32 ? reinterpret_cast<const float*>(w)[d] : to_f(reinterpret_cast<const T*>(w)[d]);
      y[i] = round_to<T>(wv * (x[i] * rs));
    }
    // rotate the first rotary_dim dims: out = bf16(bf16(y c) + bf16(rot(y) s)),
    // rot(y)_d = -y_(d+half) for d < half, y_(d-half) for half <= d < 2 half
    float o[E];
    if (half >= 32) {
      const int hi = half / 32;  // the partner sits hi elements further in the same lane
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int d = lane + 32 * i;
        if (d < 2 * half) {
          const int j = d < half ? d : d - half;
          const float pr = d < half ? -y[i + hi < E ? i + hi : i] : y[i - hi >= 0 ? i - hi : i];
          o[i] = round_to<T>(round_to<T>(y[i] * cs[j]) + round_to<T>(pr * sn[j]));
        } else {
          o[i] = y[i];
        }
      }
    } else {
      // half < 32 (a power of two): only element 0 of lanes [0, 2 half) rotates
#pragma unroll
      for (int i = 0; i < E; ++i) o[i] = y[i];
      const float partner = __shfl_xor_sync(0xffffffffu, y[0], half);
      if (lane < 2 * half) {
        const int j = lane < half ? lane : lane - half;
        const float pr = lane < half ? -partner : partner;
        o[0] = round_to<T>(round_to<T>(y[0] * cs[j]) + round_to<T>(pr * sn[j]));
      }
    }
#pragma unroll
    for (int i = 0; i < E; ++i) dst[lane + 32 * i] = from_f<T>(o[i]);
  }
}

// Vector form: lane l holds the E = D/32 contiguous elements [E l, E l + E) of a row (one 16-byte
// access at D 256 in bf16), so the rotation partner d +- half sits in lane l ^ (half / E) at the
// same position.  Needs rows aligned to E elements and half a multiple of E with half / E a power
// of two below 32 (rotary_dim = D/4 at D 64/128/256).
//
// A CTA takes TPC consecutive tokens: one preamble (cos/sin of its tokens, their pool slots) and
// one barrier for all of them, then its warps walk the TPC x (Hq + 2 Hkv) rows (row ri is head row
// ri / TPC of token ri % TPC) with a ring of PF rows in flight per warp.  The norm weights sit in
// registers, cos/sin are read as vectors, and the rotation partners of 16-bit rows cross lanes two
// per shuffle: about a third of the shared/shuffle traffic of one token per CTA.
template <int BYTES> struct VecT;
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<8> { using type = uint2; };
template <> struct VecT<16> { using type = uint4; };

template <typename V>
__device__ __forceinline__ V ld_stream(const void* p) {
  if constexpr (sizeof(V) == 16) return __ldcs(reinterpret_cast<const uint4*>(p));
  else if constexpr (sizeof(V) == 8) return __ldcs(reinterpret_cast<const uint2*>(p));
  else return __ldcs(reinterpret_cast<const unsigned int*>(p));
}

// E consecutive cos and sin values of a token from shared memory (16-byte loads when E % 4 == 0;
// the first index is a multiple of E)
template <int E>
__device__ __forceinline__ void load_cos_sin(const float* cp, const float* sp, float (&c)[E],
                                             float (&sv)[E]) {
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int k = 0; k < E / 4; ++k) {
      const float4 c4 = reinterpret_cast<const float4*>(cp)[k];
      const float4 s4 = reinterpret_cast<const float4*>(sp)[k];
      c[4 * k] = c4.x; c[4 * k + 1] = c4.y; c[4 * k + 2] = c4.z; c[4 * k + 3] = c4.w;
      sv[4 * k] = s4.x; sv[4 * k + 1] = s4.y; sv[4 * k + 2] = s4.z; sv[4 * k + 3] = s4.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) { c[e] = cp[e]; sv[e] = sp[e]; }
  }
}

template <typename T, int D, int TPC>
__global__ void __launch_bounds__(kThreads, 3) prologue_vec_kernel(tf_attn_prologue_args a) {
  constexpr int E = D / 32;
  constexpr int NW = kThreads / 32;
  constexpr int PF = 4;
  static_assert(NW % TPC == 0, "a warp serves one token");
  constexpr int RSTEP = NW / TPC;  // head rows between a warp's consecutive rows
  using V = typename VecT<E * (int)sizeof(T)>::type;
  __shared__ __align__(16) float cs[TPC][kMaxD / 2];
  __shared__ __align__(16) float sn[TPC][kMaxD / 2];
  __shared__ int64_t s_loc[TPC];
  const int64_t t0 = (int64_t)blockIdx.x * TPC;
  const int ntok = a.num_tokens - t0 < TPC ? (int)(a.num_tokens - t0) : TPC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = a.num_q_heads, Hkv = a.num_kv_heads;
  const int nrows = Hq + 2 * Hkv;
  const int d0 = lane * E;
  // warp w serves token tt = w % TPC, head rows r0, r0 + RSTEP, ... (q heads, then k, then v)
  const int tt = warp % TPC, r0 = warp / TPC;
  const bool live = tt < ntok;  // warp-uniform
  const int64_t t = t0 + tt;
  const T* q_src = reinterpret_cast<const T*>(a.q) + t * a.q_stride_tok + d0;
  const T* k_src = reinterpret_cast<const T*>(a.k) + t * a.k_stride_tok + d0;
  const T* v_src = reinterpret_cast<const T*>(a.v) + t * a.v_stride_tok + d0;
  auto load = [&](int r) -> V {
    if (!live || r >= nrows) return V();
    const T* src = r < Hq ? q_src + (int64_t)r * a.q_stride_head
                 : r < Hq + Hkv ? k_src + (int64_t)(r - Hq) * a.k_stride_head
                                : v_src + (int64_t)(r - Hq - Hkv) * a.v_stride_head;
    return ld_stream<V>(src);
  };
  // this warp's first rows are loading while the tokens' cos/sin and slots are prepared
  V ring[PF];
#pragma unroll
  for (int u = 0; u < PF; ++u) ring[u] = load(r0 + u * RSTEP);
  const int half = a.rotary_dim / 2;
  for (int j = tid; j < TPC * half; j += kThreads) {
    const int jt = j / half, jj = j - jt * half;
    if (jt >= ntok) continue;
    int prow = 0;
    if (a.pos_rows == 3) {
      if (a.mrope_interleaved) {
        const int m = jj % 3;
        if (m == 1 && jj < 3 * a.mrope_section[1]) prow = 1;
        else if (m == 2 && jj < 3 * a.mrope_section[2]) prow = 2;
      } else {
        prow = jj < a.mrope_section[0] ? 0 : (jj < a.mrope_section[0] + a.mrope_section[1] ? 1 : 2);
      }
    }
    const float f = (float)a.positions[prow * a.pos_stride + t0 + jt] * a.inv_freq[jj];
    float sf, cf;
    sincosf(f, &sf, &cf);
    cs[jt][jj] = round_to<T>(cf);
    sn[jt][jj] = round_to<T>(sf);
  }
  if (tid >= 32 && tid < 32 + TPC && tid - 32 < ntok) {
    int64_t loc = a.out_cache_loc[t0 + tid - 32];
    if (loc < 0) loc += a.num_slots;  // torch index semantics
    if (loc < 0 || loc >= a.num_slots) {
      record_err(a.err, TF_KERR_SLOT_RANGE);
      loc = -1;
    }
    s_loc[tid - 32] = loc;
  }
  float wq[E], wk[E];
  const bool wf32 = a.norm_weight_dtype == TF_DTYPE_F32;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    wq[e] = wf32 ? reinterpret_cast<const float*>(a.q_norm_weight)[d0 + e]
                 : to_f(reinterpret_cast<const T*>(a.q_norm_weight)[d0 + e]);
    wk[e] = wf32 ? reinterpret_cast<const float*>(a.k_norm_weight)[d0 + e]
                 : to_f(reinterpret_cast<const T*>(a.k_norm_weight)[d0 + e]);
  }
  __syncthreads();
  if (!live) return;
  const int64_t loc = s_loc[tt];
  T* q_dst = reinterpret_cast<T*>(a.q_out) + t * a.q_out_stride_tok + d0;
  T* k_dst = loc < 0 ? nullptr : reinterpret_cast<T*>(a.k_buffer) + loc * a.buf_stride_slot + d0;
  T* v_dst = loc < 0 ? nullptr : reinterpret_cast<T*>(a.v_buffer) + loc * a.buf_stride_slot + d0;
  const int pmask = half / E;  // rotation partner: lane ^ pmask
  const bool rotates = d0 < 2 * half, lower = d0 < half;
  const int j0 = lower ? d0 : d0 - half;
  // rotary_dim 64 at D 256 (the 0.25 partial rotation): the 32 bf16 pairs of the rotated dims sit
  // in lanes 0-7; they are spread one pair per lane for the rotation and gathered back, so the
  // rotation's roundings run on all 32 lanes instead of 8
  const bool spread = sizeof(T) == 2 && E == 8 && half == 32;
  for (int m0 = 0; r0 + m0 * RSTEP < nrows; m0 += PF) {
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int r = r0 + (m0 + u) * RSTEP;
      if (r >= nrows) break;
      const V cur = ring[u];
      ring[u] = load(r + PF * RSTEP);
      T* dst;
      if (r < Hq) {
        dst = q_dst + (int64_t)r * a.q_out_stride_head;
      } else if (loc < 0) {
        continue;
      } else if (r >= Hq + Hkv) {  // v: copied as is
        *reinterpret_cast<V*>(v_dst + (int64_t)(r - Hq - Hkv) * a.buf_stride_head) = cur;
        continue;
      } else {
        dst = k_dst + (int64_t)(r - Hq) * a.buf_stride_head;
      }
      const bool isq = r < Hq;
      V outv;
      if constexpr (sizeof(T) == 2) {
        // 16-bit rows stay in packed pairs: each rounding is one paired conversion
        constexpr int W2 = E / 2;
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(&cur);
        float x[E];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < W2; ++i) {
          x[2 * i] = unpack_lo<T>(xw[i]);
          x[2 * i + 1] = unpack_hi<T>(xw[i]);
          ss = fmaf(x[2 * i], x[2 * i], ss);
          ss = fmaf(x[2 * i + 1], x[2 * i + 1], ss);
        }
        ss = warp_sum(ss);
        const float rs = rsqrtf(ss / (float)D + a.eps);
        uint32_t yw[W2];
#pragma unroll
        for (int i = 0; i < W2; ++i)
          yw[i] = pack2_rn<T>((isq ? wq[2 * i] : wk[2 * i]) * (x[2 * i] * rs),
                              (isq ? wq[2 * i + 1] : wk[2 * i + 1]) * (x[2 * i + 1] * rs));
        uint32_t* ow = reinterpret_cast<uint32_t*>(&outv);
        if (spread) {
          if constexpr (W2 == 4) {
            // lane l takes word l % 4 of lane l / 4: dims 2l, 2l + 1; the partner pair is lane l ^ 16
            uint32_t g = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t v = __shfl_sync(0xffffffffu, yw[k], lane >> 2);
              if ((lane & 3) == k) g = v;
            }
            const uint32_t pg = __shfl_xor_sync(0xffffffffu, g, 16);
            const bool lo_half = lane < 16;
            const int jj = (2 * lane) & 31;
            const float2 c2 = *reinterpret_cast<const float2*>(&cs[tt][jj]);
            const float2 s2 = *reinterpret_cast<const float2*>(&sn[tt][jj]);
            const float p0 = unpack_lo<T>(pg), p1 = unpack_hi<T>(pg);
            const uint32_t t1 = pack2_rn<T>(unpack_lo<T>(g) * c2.x, unpack_hi<T>(g) * c2.y);
            const uint32_t t2 = pack2_rn<T>((lo_half ? -p0 : p0) * s2.x, (lo_half ? -p1 : p1) * s2.y);
            const uint32_t og = pack2_rn<T>(unpack_lo<T>(t1) + unpack_lo<T>(t2),
                                            unpack_hi<T>(t1) + unpack_hi<T>(t2));
            // lane s < 8 takes back word k from lane 4 s + k
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t v = __shfl_sync(0xffffffffu, og, (4 * lane + k) & 31);
              ow[k] = lane < 8 ? v : yw[k];
            }
          }
        } else {
          uint32_t pw[W2];
#pragma unroll
          for (int i = 0; i < W2; ++i) pw[i] = __shfl_xor_sync(0xffffffffu, yw[i], pmask);
          if (rotates) {
            float c[E], sv[E];
            load_cos_sin<E>(&cs[tt][j0], &sn[tt][j0], c, sv);
#pragma unroll
            for (int i = 0; i < W2; ++i) {
              const float p0 = unpack_lo<T>(pw[i]), p1 = unpack_hi<T>(pw[i]);
              const uint32_t t1 = pack2_rn<T>(unpack_lo<T>(yw[i]) * c[2 * i],
                                              unpack_hi<T>(yw[i]) * c[2 * i + 1]);
              const uint32_t t2 = pack2_rn<T>((lower ? -p0 : p0) * sv[2 * i],
                                              (lower ? -p1 : p1) * sv[2 * i + 1]);
              ow[i] = pack2_rn<T>(unpack_lo<T>(t1) + unpack_lo<T>(t2),
                                  unpack_hi<T>(t1) + unpack_hi<T>(t2));
            }
          } else {
#pragma unroll
            for (int i = 0; i < W2; ++i) ow[i] = yw[i];
          }
        }
      } else {
        const T* xe = reinterpret_cast<const T*>(&cur);
        float x[E], y[E], p[E];
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          x[e] = to_f(xe[e]);
          ss = fmaf(x[e], x[e], ss);
        }
        ss = warp_sum(ss);
        const float rs = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          y[e] = round_to<T>((isq ? wq[e] : wk[e]) * (x[e] * rs));
          p[e] = __shfl_xor_sync(0xffffffffu, y[e], pmask);
        }
        T* oe = reinterpret_cast<T*>(&outv);
        if (rotates) {
          float c[E], sv[E];
          load_cos_sin<E>(&cs[tt][j0], &sn[tt][j0], c, sv);
#pragma unroll
          for (int e = 0; e < E; ++e)
            oe[e] = from_f<T>(round_to<T>(round_to<T>(y[e] * c[e]) +
                                          round_to<T>((lower ? -p[e] : p[e]) * sv[e])));
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) oe[e] = from_f<T>(y[e]);
        }
      }
      *reinterpret_cast<V*>(dst) = outv;
    }
  }
}

template <typename T>
static bool vec_ok(const tf_attn_prologue_args& a) {
  const int E = a.head_dim / 32;
  const int vb = E * (int)sizeof(T);
  if (vb != 4 && vb != 8 && vb != 16) return false;
  const int half = a.rotary_dim / 2;
  if (half % E || half / E >= 32 || ((half / E) & (half / E - 1))) return false;
  auto al = [vb](const void* p) { return (reinterpret_cast<uintptr_t>(p) % vb) == 0; };
  if (!al(a.q) || !al(a.k) || !al(a.v) || !al(a.q_out) || !al(a.k_buffer) || !al(a.v_buffer))
    return false;
  const int64_t st[] = {a.q_stride_tok, a.q_stride_head, a.k_stride_tok, a.k_stride_head,
                        a.v_stride_tok, a.v_stride_head, a.q_out_stride_tok, a.q_out_stride_head,
                        a.buf_stride_slot, a.buf_stride_head};
  for (int64_t x : st)
    if (x % E) return false;
  return true;
}

template <typename T>
static cudaError_t launch_t(const tf_attn_prologue_args& a, cudaStream_t s) {
  const unsigned g = (unsigned)a.num_tokens;
  if (vec_ok<T>(a)) {
    const unsigned gv = (unsigned)((a.num_tokens + kTPC - 1) / kTPC);
    switch (a.head_dim) {
      case 64: prologue_vec_kernel<T, 64, kTPC><<<gv, kThreads, 0, s>>>(a); break;
      case 128: prologue_vec_kernel<T, 128, kTPC><<<gv, kThreads, 0, s>>>(a); break;
      default:  // 16-bit only: fp32 rows of 256 need 32 bytes per lane and take the strided form
        if constexpr (sizeof(T) == 2) prologue_vec_kernel<T, 256, kTPC><<<gv, kThreads, 0, s>>>(a);
        break;
    }
    return cudaGetLastError();
  }
  switch (a.head_dim) {
    case 64: prologue_kernel<T, 64><<<g, kThreads, 0, s>>>(a); break;
    case 128: prologue_kernel<T, 128><<<g, kThreads, 0, s>>>(a); break;
    default: prologue_kernel<T, 256><<<g, kThreads, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace prologue

bool attn_prologue_supported(const tf_attn_prologue_args& a) {
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  const int half = a.rotary_dim / 2;
  if (a.rotary_dim < 2 || a.rotary_dim % 2 || a.rotary_dim > a.head_dim) return false;
  if (half >= 32) return half % 32 == 0;
  return (half & (half - 1)) == 0;
}

cudaError_t launch_attn_prologue(const tf_attn_prologue_args& a, cudaStream_t s) {
  if (a.num_tokens == 0) return cudaSuccess;
  switch (a.dtype) {
    case TF_DTYPE_F32: return prologue::launch_t<float>(a, s);
    case TF_DTYPE_BF16: return prologue::launch_t<__nv_bfloat16>(a, s);
    default: return prologue::launch_t<__half>(a, s);
  }
}

}  // namespace tf
