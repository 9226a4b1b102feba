// a2 + a4: paged GQA flash-decoding for bf16 pools (qwen3_8/full_attention.py:215-242 and the output
// gate of :157-158), HBM-bound by design.
//
// Work decomposition (balanced split-KV).  A unit is (request b, kv head h); its keys are cut into
// tiles of 32 tokens.  All tiles of all units form one sequence (request-major, then kv head), and
// persistent CTA c (one per SM) takes the contiguous range [c*T/G, (c+1)*T/G) of it, so every SM
// streams the same number of K/V bytes whatever the spread of seq_lens.  A unit that lies inside one
// CTA range is finished in place; a unit cut by range boundaries leaves (max, sum, unnormalised O)
// partials that a combine kernel merges.  A plan kernel computes the tile prefix over requests on
// the device, so nothing about seq_lens needs to reach the host.
//
// Inside a CTA: one producer warp gathers the token rows of each tile (slot ids from req_to_token,
// 16-byte cp.async per lane, XOR-swizzled rows) into a ring of shared-memory stages, signalling each
// stage's full mbarrier with cp.async.mbarrier.arrive; four consumer warps take tiles round-robin.
// A consumer computes S^T = K.Q^T with mma.m16n8k16 (A = 16 tokens x 16 dims of K via ldmatrix,
// B = Q^T of the 8 query heads sharing the kv head), keeps an online softmax per head in registers,
// turns P into the B operand of O^T = V^T.P^T with movmatrix (8x8 transpose in registers) and
// accumulates O^T[D x 8] in registers (V^T via ldmatrix.trans).  The four warps merge through
// shared memory at the end of each unit piece.  Every mbarrier wait is bounded.
#include "common.cuh"
#include "launch.h"

namespace tf {
namespace dec {

constexpr int kTileTok = 32;
constexpr int kConsumers = 4;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kHeads = 8;  // n of the mma tiles: query heads per kv head, padded to 8
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileBytes = kTileTok * kRowBytes;  // K (or V) rows of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = D == 256 ? 5 : 8;
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  static constexpr int kRowsPerIssue = 32 / kChunks;
  static constexpr int kOStride = D + 4;  // merge buffer row stride (floats), bank-conflict free
  static constexpr size_t kStagesBytes = (size_t)kStages * kStageBytes;
  static constexpr size_t kMergeBytes = (size_t)kConsumers * kHeads * kOStride * 4 +
                                        2 * kConsumers * kHeads * 4;
  static constexpr size_t kSmem = kStagesBytes + kMergeBytes + 2 * kStages * 8 + 64;
};

struct Ws {
  int32_t* status;
  int32_t* tile_start;  // [B+1]
  float* part_ml;       // [2*nctas][kHeads][2]  (max in log2 domain, sum)
  float* part_o;        // [2*nctas][kHeads][D]
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

__host__ __device__ inline Ws carve(void* base, int B, int nctas, int D) {
  char* p = (char*)base;
  Ws w;
  w.status = (int32_t*)p;
  p += 256;
  w.tile_start = (int32_t*)p;
  p += align256((size_t)(B + 1) * 4);
  w.part_ml = (float*)p;
  p += align256((size_t)2 * nctas * kHeads * 2 * 4);
  w.part_o = (float*)p;
  return w;
}

inline size_t ws_bytes(int B, int nctas, int D) {
  return 256 + align256((size_t)(B + 1) * 4) + align256((size_t)2 * nctas * kHeads * 2 * 4) +
         (size_t)2 * nctas * kHeads * D * 4;
}

// ---------------------------------------------------------------------------------------------
// plan: tile_start[b] = sum_{b'<b} ceil(seq_lens[b'] / 32)
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) plan_kernel(const int64_t* seq_lens, int B,
                                                    int32_t* tile_start) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int b0 = 0; b0 < B; b0 += 1024) {
    const int b = b0 + tid;
    int64_t L = b < B ? seq_lens[b] : 0;
    if (L < 0) L = 0;
    int32_t v = (int32_t)((L + kTileTok - 1) / kTileTok);
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int32_t w = warp_tot[lane];
      int32_t wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int32_t y = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += y;
      }
      warp_tot[lane] = wi - w;  // exclusive
    }
    __syncthreads();
    const int32_t excl = carry + warp_tot[warp] + incl - v;
    if (b < B) tile_start[b] = excl;
    __syncthreads();
    if (tid == 1023) carry = excl + v;
    __syncthreads();
  }
  if (tid == 0) tile_start[B] = carry;
}

// ---------------------------------------------------------------------------------------------
// walking the tile sequence
// ---------------------------------------------------------------------------------------------
struct Piece {
  int b, h, t0, n;  // tiles [t0, t0+n) of unit (b, h)
  int nt;           // tiles of the whole unit
  int64_t g_start;  // global index of the piece's first tile
};

struct Walker {
  const int32_t* ts;
  int B, Hkv;
  int64_t g, g1;
  int b;
  __device__ void init(const int32_t* ts_, int B_, int Hkv_, int64_t g0, int64_t g1_) {
    ts = ts_; B = B_; Hkv = Hkv_; g = g0; g1 = g1_;
    // first b with ts[b+1]*Hkv > g0
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((int64_t)ts[mid + 1] * Hkv > g0) hi = mid; else lo = mid + 1;
    }
    b = lo;
  }
  __device__ bool next(Piece& p) {
    if (g >= g1) return false;
    while ((int64_t)ts[b + 1] * Hkv <= g) ++b;
    const int nt = ts[b + 1] - ts[b];
    const int64_t within = g - (int64_t)ts[b] * Hkv;
    p.b = b;
    p.h = (int)(within / nt);
    p.t0 = (int)(within - (int64_t)p.h * nt);
    const int64_t rem = g1 - g;
    p.n = (int)(rem < nt - p.t0 ? rem : nt - p.t0);
    p.nt = nt;
    p.g_start = g;
    g += p.n;
    return true;
  }
};

__device__ __forceinline__ int64_t cta_range(int c, int64_t total, int nctas) {
  return (int64_t)c * total / nctas;
}

// ---------------------------------------------------------------------------------------------
// tensor-core helpers (legacy warp-level mma; operands staged by cp.async + ldmatrix)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---------------------------------------------------------------------------------------------
// main kernel
// ---------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(tf_paged_attn_args a, Ws ws, int nctas_launched) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* stages = smem;
  float* o_s = reinterpret_cast<float*>(smem + C::kStagesBytes);       // [4][8][kOStride]
  float* m_s = o_s + kConsumers * kHeads * C::kOStride;                // [4][8]
  float* l_s = m_s + kConsumers * kHeads;                              // [4][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(l_s + kConsumers * kHeads);
  uint64_t* empty = full + C::kStages;
  volatile int* aborted = reinterpret_cast<volatile int*>(empty + C::kStages);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = a.batch_size, Hkv = a.num_kv_heads;
  const int G = a.num_q_heads / Hkv;
  int32_t* err = a.err ? a.err : ws.status;

  const int64_t total = (int64_t)ws.tile_start[B] * Hkv;
  const int nctas = (int64_t)nctas_launched < total ? nctas_launched : (int)total;
  const int c = blockIdx.x;
  if (c >= nctas) return;
  const int64_t g0 = cta_range(c, total, nctas), g1 = cta_range(c + 1, total, nctas);

  if (tid == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 32);  // one cp.async arrival per producer lane
      mbar_init(&empty[s], 1);  // the consumer warp that read the stage
    }
    *aborted = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const uint32_t stage0 = smem_u32(stages);

  if (warp == kConsumers) {
    // ===================================== producer =====================================
    Walker wk;
    wk.init(ws.tile_start, B, Hkv, g0, g1);
    Piece p;
    int i = 0;
    const char* kb = (const char*)a.k_buffer;
    const char* vb = (const char*)a.v_buffer;
    const int row_in = lane / C::kChunks, chunk = lane % C::kChunks;
    bool ok = true;
    while (ok && wk.next(p)) {
      int64_t row = a.req_pool_indices[p.b];
      if (row < 0 || row >= a.r2t_rows) { record_err(err, TF_KERR_REQ_RANGE); row = 0; }
      const int64_t* r2t = a.req_to_token + row * a.r2t_stride;
      const int64_t L = a.seq_lens[p.b];
      const int64_t head_off = (int64_t)p.h * a.kv_stride_head * 2 + chunk * 16;
      // slot ids of the first tile, then one tile of look-ahead
      int64_t pos = (int64_t)p.t0 * kTileTok + lane;
      int64_t raw_next = r2t[pos < L ? pos : (int64_t)p.t0 * kTileTok];
      for (int tt = 0; tt < p.n; ++tt, ++i) {
        const int64_t raw = raw_next;
        if (tt + 1 < p.n) {
          const int64_t base = (int64_t)(p.t0 + tt + 1) * kTileTok;
          raw_next = r2t[base + lane < L ? base + lane : base];
        }
        const int64_t slot = resolve_slot(raw, a.num_slots, a.slot_mode, err);
        const int s = i % C::kStages;
        if (i >= C::kStages) {
          if (!mbar_wait(&empty[s], ((i / C::kStages) - 1) & 1)) {
            record_err(err, TF_KERR_TIMEOUT);
            ok = false;
            break;
          }
        }
        const uint32_t kdst = stage0 + s * C::kStageBytes;
#pragma unroll 4
        for (int r = 0; r < kTileTok; r += C::kRowsPerIssue) {
          const int rr = r + row_in;
          const int64_t sl = __shfl_sync(0xffffffffu, slot, rr);
          const int64_t off = sl * a.kv_stride_slot * 2 + head_off;
          const uint32_t dst = kdst + rr * C::kRowBytes + ((chunk ^ (rr & 7)) << 4);
          cp_async16(dst, kb + off);
          cp_async16(dst + C::kTileBytes, vb + off);
        }
        cp_async_arrive_noinc(&full[s]);
      }
    }
    cp_async_wait_all();
    return;
  }

  // ====================================== consumers ======================================
  const int gq = lane >> 2, tq = lane & 3;  // mma groupID / thread-in-group
  const float scale_log2 = a.scale * kLog2e;
  Walker wk;
  wk.init(ws.tile_start, B, Hkv, g0, g1);
  Piece p;
  int i_base = 0;
  const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(a.q);
  while (wk.next(p)) {
    // Q^T fragments of the query heads of kv head p.h (token index == request index in decode)
    uint32_t qf[D / 16][2];
    {
      const bool live = gq < G;
      const __nv_bfloat16* qrow =
          qg + (int64_t)p.b * a.q_stride_tok + (int64_t)(p.h * G + (live ? gq : 0)) * a.q_stride_head;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        qf[kk][0] = live ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * tq) : 0u;
        qf[kk][1] = live ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * tq + 8) : 0u;
      }
    }
    float acc[D / 16][4];
#pragma unroll
    for (int md = 0; md < D / 16; ++md) acc[md][0] = acc[md][1] = acc[md][2] = acc[md][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int64_t L = a.seq_lens[p.b];

    const int first = i_base + (((warp - i_base) % kConsumers) + kConsumers) % kConsumers;
    for (int i = first; i < i_base + p.n; i += kConsumers) {
      const int s = i % C::kStages;
      if (*aborted) continue;
      if (!mbar_wait(&full[s], (i / C::kStages) & 1)) {
        if (lane == 0) { record_err(err, TF_KERR_TIMEOUT); *aborted = 1; }
        continue;
      }
      const uint32_t kbase = stage0 + s * C::kStageBytes;
      const uint32_t vbase = kbase + C::kTileBytes;
      const int64_t tok0 = (int64_t)(p.t0 + (i - i_base)) * kTileTok;

      float sc[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
        const int row = mt * 16 + (lane & 15);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int ch = kk * 2 + (lane >> 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kbase + row * C::kRowBytes + ((ch ^ (row & 7)) << 4), a0, a1, a2, a3);
          mma_bf16(sc[mt], a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
        }
      }
      // scale, mask, online softmax (columns 2tq, 2tq+1 are query heads; rows are tokens)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const bool v_lo = tok0 + mt * 16 + gq < L;
        const bool v_hi = tok0 + mt * 16 + gq + 8 < L;
        sc[mt][0] = v_lo ? sc[mt][0] * scale_log2 : -INFINITY;
        sc[mt][1] = v_lo ? sc[mt][1] * scale_log2 : -INFINITY;
        sc[mt][2] = v_hi ? sc[mt][2] * scale_log2 : -INFINITY;
        sc[mt][3] = v_hi ? sc[mt][3] * scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(sc[mt][0], sc[mt][2]));
        mx1 = fmaxf(mx1, fmaxf(sc[mt][1], sc[mt][3]));
      }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      l0 *= al0;
      l1 *= al1;
      uint32_t pb[2][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float p0 = exp2f(sc[mt][0] - mn0), p1 = exp2f(sc[mt][1] - mn1);
        const float p2 = exp2f(sc[mt][2] - mn0), p3 = exp2f(sc[mt][3] - mn1);
        l0 += p0 + p2;
        l1 += p1 + p3;
        pb[mt][0] = movmatrix_t(pack_bf16(p0, p1));
        pb[mt][1] = movmatrix_t(pack_bf16(p2, p3));
      }
#pragma unroll
      for (int md = 0; md < D / 16; ++md) {
        acc[md][0] *= al0;
        acc[md][1] *= al1;
        acc[md][2] *= al0;
        acc[md][3] *= al1;
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int row = mt * 16 + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
        for (int md = 0; md < D / 16; ++md) {
          const int ch = md * 2 + ((lane >> 3) & 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vbase + row * C::kRowBytes + ((ch ^ (row & 7)) << 4), a0, a1, a2, a3);
          mma_bf16(acc[md], a0, a1, a2, a3, pb[mt][0], pb[mt][1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    i_base += p.n;

    // ---------------- merge the four consumer warps of this piece ----------------
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (gq == 0) {
      m_s[warp * kHeads + 2 * tq] = m0;
      m_s[warp * kHeads + 2 * tq + 1] = m1;
      l_s[warp * kHeads + 2 * tq] = l0;
      l_s[warp * kHeads + 2 * tq + 1] = l1;
    }
    named_barrier(1, 32 * kConsumers);
    float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) {
      M0 = fmaxf(M0, m_s[w * kHeads + 2 * tq]);
      M1 = fmaxf(M1, m_s[w * kHeads + 2 * tq + 1]);
    }
    const float f0 = m0 == -INFINITY ? 0.f : exp2f(m0 - M0);
    const float f1 = m1 == -INFINITY ? 0.f : exp2f(m1 - M1);
    float* ow = o_s + warp * kHeads * C::kOStride;
#pragma unroll
    for (int md = 0; md < D / 16; ++md) {
      ow[(2 * tq) * C::kOStride + md * 16 + gq] = acc[md][0] * f0;
      ow[(2 * tq + 1) * C::kOStride + md * 16 + gq] = acc[md][1] * f1;
      ow[(2 * tq) * C::kOStride + md * 16 + gq + 8] = acc[md][2] * f0;
      ow[(2 * tq + 1) * C::kOStride + md * 16 + gq + 8] = acc[md][3] * f1;
    }
    named_barrier(1, 32 * kConsumers);
    const bool complete = (p.t0 == 0 && p.n == p.nt);
    const int pslot = 2 * c + (p.g_start == g0 ? 0 : 1);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
    for (int e = tid; e < G * D; e += 32 * kConsumers) {
      const int hd = e / D, d = e - hd * D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, m_s[w * kHeads + hd]);
      float Ls = 0.f, o = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float mw = m_s[w * kHeads + hd];
        Ls += mw == -INFINITY ? 0.f : l_s[w * kHeads + hd] * exp2f(mw - M);
        o += o_s[(w * kHeads + hd) * C::kOStride + d];
      }
      if (complete) {
        const int hq = p.h * G + hd;
        float r = round_to<__nv_bfloat16>(o / Ls);
        if (a.gate_mode != TF_GATE_NONE && gate != nullptr)
          r = apply_gate<__nv_bfloat16>(
              r, to_f(gate[(int64_t)p.b * a.gate_stride_tok + (int64_t)hq * a.gate_stride_head + d]),
              a.gate_mode);
        out[(int64_t)p.b * a.out_stride_tok + (int64_t)hq * a.out_stride_head + d] =
            __float2bfloat16_rn(r);
      } else {
        ws.part_o[((int64_t)pslot * kHeads + hd) * D + d] = o;
        if (d == 0) {
          ws.part_ml[(pslot * kHeads + hd) * 2 + 0] = M;
          ws.part_ml[(pslot * kHeads + hd) * 2 + 1] = Ls;
        }
      }
    }
    named_barrier(1, 32 * kConsumers);
  }
}

// ---------------------------------------------------------------------------------------------
// combine: units cut by CTA range boundaries
// ---------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) combine_kernel(tf_paged_attn_args a, Ws ws,
                                                      int nctas_launched) {
  const int B = a.batch_size, Hkv = a.num_kv_heads;
  const int G = a.num_q_heads / Hkv;
  const int b = blockIdx.x / Hkv, h = blockIdx.x - (blockIdx.x / Hkv) * Hkv;
  const int64_t total = (int64_t)ws.tile_start[B] * Hkv;
  const int nctas = (int64_t)nctas_launched < total ? nctas_launched : (int)total;
  const int nt = ws.tile_start[b + 1] - ws.tile_start[b];
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
  if (nt == 0) {  // no keys: softmax over an empty row is NaN in the reference as well
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
      const int hd = e / D, d = e - hd * D;
      out[(int64_t)b * a.out_stride_tok + (int64_t)(h * G + hd) * a.out_stride_head + d] =
          __float2bfloat16_rn(NAN);
    }
    return;
  }
  const int64_t su = (int64_t)ws.tile_start[b] * Hkv + (int64_t)h * nt, eu = su + nt;
  const int c0 = (int)(((su + 1) * nctas - 1) / total);
  const int c1 = (int)((eu * nctas - 1) / total);
  if (c0 == c1) return;  // finished inside one CTA
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int hd = e / D, d = e - hd * D;
    float M = -INFINITY;
    for (int cc = c0; cc <= c1; ++cc) {
      const int64_t rc = cta_range(cc, total, nctas);
      const int sl = 2 * cc + ((su > rc ? su : rc) == rc ? 0 : 1);
      M = fmaxf(M, ws.part_ml[(sl * kHeads + hd) * 2]);
    }
    float Ls = 0.f, o = 0.f;
    for (int cc = c0; cc <= c1; ++cc) {
      const int64_t rc = cta_range(cc, total, nctas);
      const int sl = 2 * cc + ((su > rc ? su : rc) == rc ? 0 : 1);
      const float mw = ws.part_ml[(sl * kHeads + hd) * 2];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
      Ls += ws.part_ml[(sl * kHeads + hd) * 2 + 1] * f;
      o += ws.part_o[((int64_t)sl * kHeads + hd) * D + d] * f;
    }
    const int hq = h * G + hd;
    float r = round_to<__nv_bfloat16>(o / Ls);
    if (a.gate_mode != TF_GATE_NONE && gate != nullptr)
      r = apply_gate<__nv_bfloat16>(
          r, to_f(gate[(int64_t)b * a.gate_stride_tok + (int64_t)hq * a.gate_stride_head + d]),
          a.gate_mode);
    out[(int64_t)b * a.out_stride_tok + (int64_t)hq * a.out_stride_head + d] = __float2bfloat16_rn(r);
  }
}

template <int D>
static cudaError_t launch_d(const tf_paged_attn_args& a, void* wsp, int nctas, cudaStream_t s) {
  Ws ws = carve(wsp, a.batch_size, nctas, D);
  cudaError_t e = cudaFuncSetAttribute(decode_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Cfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  plan_kernel<<<1, 1024, 0, s>>>(a.seq_lens, a.batch_size, ws.tile_start);
  decode_kernel<D><<<nctas, kThreads, Cfg<D>::kSmem, s>>>(a, ws, nctas);
  combine_kernel<D><<<a.batch_size * a.num_kv_heads, 256, 0, s>>>(a, ws, nctas);
  return cudaGetLastError();
}

}  // namespace dec

bool paged_decode_mma_supported(const tf_paged_attn_args& a) {
  if (a.dtype != TF_DTYPE_BF16) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  const int G = a.num_q_heads / a.num_kv_heads;
  if (G < 1 || G > dec::kHeads) return false;
  auto al = [](const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
  if (!al(a.k_buffer, 16) || !al(a.v_buffer, 16)) return false;
  if ((a.kv_stride_slot * 2) % 16 != 0 || (a.kv_stride_head * 2) % 16 != 0) return false;
  if (!al(a.q, 4) || (a.q_stride_tok % 2) != 0 || (a.q_stride_head % 2) != 0) return false;
  return true;
}

size_t paged_decode_mma_workspace(const tf_paged_attn_args& a, int num_sms) {
  return dec::ws_bytes(a.batch_size, num_sms, a.head_dim);
}

cudaError_t launch_paged_decode_mma(const tf_paged_attn_args& a, void* ws, size_t ws_bytes,
                                    int num_sms, cudaStream_t s) {
  (void)ws_bytes;
  if (a.batch_size == 0) return cudaSuccess;
  switch (a.head_dim) {
    case 64: return dec::launch_d<64>(a, ws, num_sms, s);
    case 128: return dec::launch_d<128>(a, ws, num_sms, s);
    default: return dec::launch_d<256>(a, ws, num_sms, s);
  }
}

}  // namespace tf
