// a2 + a4: paged GQA flash-decoding for bf16 pools (qwen3_8/full_attention.py:215-242 and the output
// gate of :157-158), HBM-bound by design.
//
// Work decomposition (balanced split-KV).  A unit is (request b, kv head h); its keys are cut into
// tiles of 16 tokens.  All tiles of all units form one sequence (request-major, then kv head), and
// persistent CTA c (one per SM) takes the contiguous range [c*T/G, (c+1)*T/G) of it, so every SM
// streams the same number of K/V bytes whatever the spread of seq_lens.  A unit that lies inside one
// CTA range is finished in place; a unit cut by range boundaries leaves (max, sum, unnormalised O)
// partials that a combine kernel merges.  A plan kernel computes the tile prefix over requests on
// the device, so nothing about seq_lens needs to reach the host.
//
// Inside a CTA the eight warps take the tiles of a unit round-robin and stream K/V rows straight
// from HBM into registers with 16-byte loads (no shared-memory staging: many warps with loads in
// flight is what saturates HBM for 512-byte random rows), one tile ahead, slot ids two tiles ahead.
// The tensor cores consume the loaded registers directly:
//   S^T = K.Q^T   mma.m16n8k16, A = 16 tokens x 16 dims of K.  The reduction over dims may visit
//                 the dims in any order as long as Q^T uses the same order, so the k-step order is
//                 chosen such that a thread's 16-byte load (8 consecutive dims of one token) IS its
//                 A fragment for two k-steps: k-step 2j takes dims 32j+8t+{0,1 | 2,3}, k-step 2j+1
//                 dims 32j+8t+{4,5 | 6,7} (t = lane%4); Q^T is read from shared memory in the same
//                 order.  B = Q^T of the 8 query heads sharing the kv head (GQA packed in n).
//   O^T = V^T.P^T A = V^T, 16 dims x 16 tokens.  Each 32-bit word of a V load is one row of an 8x8
//                 (token x dim-pair) matrix fragment; movmatrix.trans turns it into the A fragment of
//                 V^T for a dim permutation phi_c(g) = 32j + 8(g>>1) + 2c + (g&1), undone when the
//                 warps merge.  P^T (B operand) comes from the S^T accumulator through movmatrix.
// Online softmax per query head in registers; the eight warps merge through shared memory at the
// end of each unit piece.
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace tf {
namespace dec {

constexpr int kTileTok = 16;
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kHeads = 8;  // n of the mma tiles: query heads per kv head, padded to 8
constexpr float kLog2e = 1.4426950408889634f;

constexpr int kMaxCachedReqs = 256;

struct ReqCache {
  int bf, n;  // cached requests [bf, bf + n)
  int32_t ts[kMaxCachedReqs + 1];
  int64_t row_off[kMaxCachedReqs];  // req_pool_indices[b] * r2t_stride (validated)
  int64_t len[kMaxCachedReqs];
};

template <int D>
struct Cfg {
  static constexpr int kBlocks = D / 32;  // 32-dim blocks
  static constexpr int kQStride = D + 8;  // bf16 per q_s row: +16 B keeps LDS.128 conflict-free
  static constexpr int kOStride = D + 4;  // floats per merge row
  static constexpr size_t kQBytes = (size_t)kHeads * kQStride * 2;
  static constexpr size_t kMergeBytes = (size_t)kWarps * kHeads * kOStride * 4 +
                                        2 * (size_t)kWarps * kHeads * 4;
  static constexpr size_t kCacheOff = (kQBytes + kMergeBytes + 15) & ~(size_t)15;
  static constexpr size_t kSmem = kCacheOff + sizeof(ReqCache);
};

struct Ws {
  int32_t* status;
  int64_t* cta_g;       // [nctas+1] first tile of each CTA's range (the last entry: the total)
  int32_t* cta_b;       // [nctas][2] first and last request a CTA's range touches
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
  w.cta_g = (int64_t*)p;
  p += align256((size_t)(nctas + 1) * 8);
  w.cta_b = (int32_t*)p;
  p += align256((size_t)2 * nctas * 4);
  w.tile_start = (int32_t*)p;
  p += align256((size_t)(B + 1) * 4);
  w.part_ml = (float*)p;
  p += align256((size_t)2 * nctas * kHeads * 2 * 4);
  w.part_o = (float*)p;
  return w;
}

inline size_t ws_bytes(int B, int nctas, int D) {
  return 256 + align256((size_t)(nctas + 1) * 8) + align256((size_t)2 * nctas * 4) +
         align256((size_t)(B + 1) * 4) + align256((size_t)2 * nctas * kHeads * 2 * 4) +
         (size_t)2 * nctas * kHeads * D * 4;
}

// ---------------------------------------------------------------------------------------------
// plan: tile_start[b] = sum_{b'<b} ceil(seq_lens[b'] / kTileTok), then the CTAs' ranges.
//
// The work is the sequence of (request, kv head) units in request order, each ceil(len / kTileTok)
// tiles; a CTA takes a contiguous range of it, and a unit cut by range boundaries is merged by the
// combine kernel.  Besides its tiles, every piece of a unit that a CTA runs costs a fixed amount:
// its Q rows, the first slot and K/V round trips and the cross-warp epilogue (measured on config 2:
// CTA time = 290 us + 10.8 us per piece at 944 tiles, i.e. a piece ~ 35 tiles; 8.1 us ~ 25 tiles
// on the heads of one rank of four).  Ranges of equal tile counts therefore finish up to 25% apart
// when one CTA's range holds many short requests; the plan balances tiles + kPieceCost per unit
// instead.  Boundaries are strictly increasing (every CTA has at least one tile).  Batches of more
// than kPlanSmemReqs requests keep equal tile counts.
// ---------------------------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanSmemReqs = 8192;
constexpr int kPlanMaxCtas = kPlanThreads - 1;  // one thread per boundary in the fix-up scan
// kPieceCost in tiles: 32 at head_dim 256 (between the two fits above); smaller heads make a tile
// cheaper and leave most of a piece's latency-bound cost, so it is set higher there (48 at 128,
// 64 at 64: scaled, not measured)
template <int D> struct PieceCost { static constexpr int64_t v = D >= 256 ? 32 : (D >= 128 ? 48 : 64); };
// The decode CTA that the plan kernel's SM receives starts when the plan ends (the other SMs take
// theirs at once: CTAs are dispatched in index order, so it is the last one): the last range is
// shortened by about the plan's duration in tiles (4-5 us, at 0.31-0.38 us per tile).
constexpr int64_t kPlanLagTiles = 12;

// first b with ts[b+1] * Hkv > g (b in [0, B-1])
__device__ int first_req_after(const int32_t* ts, int B, int Hkv, int64_t g) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((int64_t)ts[mid + 1] * Hkv > g) hi = mid; else lo = mid + 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int64_t* seq_lens, int B,
                                                            int64_t max_len, int Hkv,
                                                            int nctas_launched, int64_t piece_cost,
                                                            Ws ws) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  __shared__ int32_t ts_s[kPlanSmemReqs + 1];
  __shared__ int64_t cg[kPlanMaxCtas + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the decode grid may be launched now: its CTAs wait for this grid before reading the plan
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const bool small = B <= kPlanSmemReqs;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int b0 = 0; b0 < B; b0 += kPlanThreads) {
    const int b = b0 + tid;
    int64_t L = b < B ? seq_lens[b] : 0;
    if (L < 0) L = 0;
    if (L > max_len) L = max_len;
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
    if (b < B) {
      ws.tile_start[b] = excl;
      if (small) ts_s[b] = excl;
    }
    __syncthreads();
    if (tid == kPlanThreads - 1) carry = excl + v;
    __syncthreads();
  }
  if (tid == 0) {
    ws.tile_start[B] = carry;
    if (small) ts_s[B] = carry;
  }
  __syncthreads();  // the tile starts (shared and, for this CTA, global) are complete
  const int32_t* ts = small ? ts_s : ws.tile_start;
  const int64_t total = (int64_t)carry * Hkv;
  const int nctas = (int64_t)nctas_launched < total ? nctas_launched : (int)total;
  if (nctas <= 0) return;
  const int64_t beta = small ? piece_cost : 0;
  const int64_t U = (int64_t)B * Hkv;
  const int64_t ctot = total + beta * U;
  const int64_t lag = small ? kPlanLagTiles : 0;
  auto unit_start = [&](int64_t u) -> int64_t {  // first tile of unit u (u < 2^31 here: B is small)
    const int b = (int)u / Hkv, h = (int)u - b * Hkv;
    return (int64_t)ts[b] * Hkv + (int64_t)h * (ts[b + 1] - ts[b]);
  };
  for (int c = tid; c <= nctas; c += kPlanThreads) {
    int64_t g;
    if (c == nctas) {
      g = total;
    } else if (beta == 0) {
      g = (int64_t)c * total / nctas;
    } else {
      // cost position x: the unit u whose [cost start, next cost start) holds it, where a unit's
      // cost start is its first tile + beta * u; its first beta of cost is the piece's fixed part
      const int64_t x = (int64_t)c * (ctot + lag) / nctas;
      int64_t lo = 0, hi = U - 1;
      while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (unit_start(mid) + beta * mid <= x) lo = mid; else hi = mid - 1;
      }
      const int b = (int)lo / Hkv;
      const int64_t gs = unit_start(lo), nt = ts[b + 1] - ts[b];
      int64_t off = x - gs - beta * lo - beta;
      off = off < 0 ? 0 : (off > nt ? nt : off);
      g = gs + off;
    }
    cg[c] = g;
  }
  __syncthreads();
  {  // strictly increasing, every CTA at least one tile: f[c] = c + max_{k <= c}(cg[k] - k) (a
     // prefix maximum; cg[0] = 0), then min(f[c], total - nctas + c), and cg[nctas] = total
    __shared__ int64_t wmax[32];
    const int c = tid;
    int64_t v = c <= nctas ? cg[c] - c : INT64_MIN;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v = v > y ? v : y;
    }
    if (lane == 31) wmax[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int64_t wv = wmax[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, wv, o);
        if (lane >= o) wv = wv > y ? wv : y;
      }
      const int64_t prev = __shfl_up_sync(0xffffffffu, wv, 1);
      wmax[lane] = lane == 0 ? INT64_MIN : prev;  // max over the warps before this one
    }
    __syncthreads();
    if (c <= nctas) {
      const int64_t before = wmax[warp];
      const int64_t f = (int64_t)c + (v > before ? v : before);
      const int64_t cap = total - nctas + c;
      cg[c] = c == nctas ? total : (f < cap ? f : cap);
    }
  }
  __syncthreads();
  for (int c = tid; c <= nctas; c += kPlanThreads) {
    ws.cta_g[c] = cg[c];
    if (c < nctas) {
      ws.cta_b[2 * c] = first_req_after(ts, B, Hkv, cg[c]);
      ws.cta_b[2 * c + 1] = first_req_after(ts, B, Hkv, cg[c + 1] - 1);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// walking the tile sequence.  The per-request metadata a CTA needs (tile starts, req_to_token row,
// seq_len) is copied to shared memory once at kernel start, so the walkers never wait on global
// memory; only requests beyond kMaxCachedReqs (a CTA spanning that many requests) are read from
// global memory.
// ---------------------------------------------------------------------------------------------
struct Meta {
  const ReqCache* c;
  const int32_t* g_ts;
  const tf_paged_attn_args* a;
  int32_t* err;
  __device__ __forceinline__ int32_t ts(int b) const {
    const int i = b - c->bf;
    return (i >= 0 && i <= c->n) ? c->ts[i] : g_ts[b];
  }
  __device__ __forceinline__ int64_t row_off(int b) const {
    const int i = b - c->bf;
    if (i >= 0 && i < c->n) return c->row_off[i];
    int64_t r = a->req_pool_indices[b];
    if (r < 0 || r >= a->r2t_rows) { record_err(err, TF_KERR_REQ_RANGE); r = 0; }
    return r * a->r2t_stride;
  }
  __device__ __forceinline__ int64_t len(int b) const {
    const int i = b - c->bf;
    if (i >= 0 && i < c->n) return c->len[i];
    const int64_t len = a->seq_lens[b];
    return len < a->r2t_cols ? len : a->r2t_cols;
  }
};

struct Piece {
  int b, h, t0, n;  // tiles [t0, t0+n) of unit (b, h)
  int nt;           // tiles of the whole unit
  int64_t g_start;  // global index of the piece's first tile
};

struct Walker {
  int Hkv;
  int64_t g, g1;
  int b;
  __device__ void init(int b0, int Hkv_, int64_t g0, int64_t g1_) {
    Hkv = Hkv_; g = g0; g1 = g1_; b = b0;
  }
  __device__ bool next(const Meta& m, Piece& p) {
    if (g >= g1) return false;
    while ((int64_t)m.ts(b + 1) * Hkv <= g) ++b;
    const int tsb = m.ts(b);
    const int nt = m.ts(b + 1) - tsb;
    const int64_t within = g - (int64_t)tsb * Hkv;
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

// the CTA whose range [cg[c], cg[c+1]) holds tile g (cg strictly increasing, cg[0] = 0)
__device__ __forceinline__ int cta_of(const int64_t* cg, int nctas, int64_t g) {
  int lo = 0, hi = nctas - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cg[mid] <= g) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ---------------------------------------------------------------------------------------------
// tensor-core helpers (legacy warp-level mma; operands staged by cp.async + ldmatrix)
// ---------------------------------------------------------------------------------------------
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
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t word(const uint4& v, int c) {
  return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(tf_paged_attn_args a, Ws ws, int nctas_launched) {
  using C = Cfg<D>;
  constexpr int NB = C::kBlocks;
  extern __shared__ __align__(128) unsigned char smem[];
  // This grid is a programmatic dependent of the plan kernel: the plan (and, through stream order,
  // every earlier launch such as the KV store) is complete and visible after this wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The combine kernel may be launched once every CTA of this grid has passed the wait above (all
  // are resident: one per SM), so it may read the plan at once; its CTAs take an SM only when a
  // CTA here has exited, and wait for this grid's completion before they read its partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(smem);             // [8][kQStride]
  float* o_s = reinterpret_cast<float*>(smem + C::kQBytes);                  // [8 warps][8][kOStride]
  float* m_s = o_s + kWarps * kHeads * C::kOStride;                          // [8][8]
  float* l_s = m_s + kWarps * kHeads;                                        // [8][8]
  ReqCache* rc = reinterpret_cast<ReqCache*>(smem + C::kCacheOff);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;  // mma groupID / thread-in-group
  const int B = a.batch_size, Hkv = a.num_kv_heads;
  const int G = a.num_q_heads / Hkv;
  int32_t* err = a.err ? a.err : ws.status;

  const int64_t total = (int64_t)ws.tile_start[B] * Hkv;
  const int nctas = (int64_t)nctas_launched < total ? nctas_launched : (int)total;
  const int c = blockIdx.x;
  if (c >= nctas) return;
  const int64_t g0 = ws.cta_g[c], g1 = ws.cta_g[c + 1];  // the plan's range and its requests

  if (tid == 0) {
    const int bf = ws.cta_b[2 * c], bl = ws.cta_b[2 * c + 1];
    rc->bf = bf;
    rc->n = min(bl - bf + 1, kMaxCachedReqs);
  }
  __syncthreads();
  for (int i = tid; i <= rc->n; i += kThreads) {  // metadata of the requests this CTA spans
    const int b = rc->bf + i;
    rc->ts[i] = ws.tile_start[b];
    if (i < rc->n) {
      int64_t r = a.req_pool_indices[b];
      if (r < 0 || r >= a.r2t_rows) { record_err(err, TF_KERR_REQ_RANGE); r = 0; }
      rc->row_off[i] = r * a.r2t_stride;
      int64_t len = a.seq_lens[b];
      if (len > a.r2t_cols) { record_err(err, TF_KERR_SLOT_RANGE); len = a.r2t_cols; }
      rc->len[i] = len;
    }
  }
  __syncthreads();
  const Meta meta{rc, ws.tile_start, &a, err};

  const float scale_log2 = a.scale * kLog2e;
  const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(a.q);
  const int64_t* r2t = a.req_to_token;
  Walker wk;
  wk.init(rc->bf, Hkv, g0, g1);
  Piece p;
  while (wk.next(meta, p)) {
    // Q of the query heads of kv head p.h (token index == request index in decode); padded heads 0
    for (int e = tid; e < kHeads * D; e += kThreads) {
      const int hd = e / D, d = e - hd * D;
      q_s[hd * C::kQStride + d] =
          hd < G ? qg[(int64_t)p.b * a.q_stride_tok + (int64_t)(p.h * G + hd) * a.q_stride_head + d]
                 : __float2bfloat16_rn(0.f);
    }
    __syncthreads();
    const int64_t L = meta.len(p.b);
    const int64_t roff = meta.row_off(p.b);
    const char* kbase = (const char*)a.k_buffer + (int64_t)p.h * a.kv_stride_head * 2;
    const char* vbase = (const char*)a.v_buffer + (int64_t)p.h * a.kv_stride_head * 2;
    const int64_t sstride = a.kv_stride_slot * 2;

    float acc[NB][2][4];
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) acc[j][q2][0] = acc[j][q2][1] = acc[j][q2][2] = acc[j][q2][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // raw req_to_token entries of tokens g and g+8 of a tile (positions clamped into the request)
    auto raw_slots = [&](int tile, int64_t& s0, int64_t& s1) {
      const int64_t base = (int64_t)tile * kTileTok + gq;
      s0 = r2t[roff + (base < L ? base : L - 1)];
      s1 = r2t[roff + (base + 8 < L ? base + 8 : L - 1)];
    };
    uint4 kr[2][NB], vr[2][NB];
    auto load_rows = [&](const char* basep, int64_t s0, int64_t s1, uint4 (&dst)[2][NB]) {
      const char* p0 = basep + s0 * sstride;
      const char* p1 = basep + s1 * sstride;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        dst[0][j] = ld_stream(p0 + (4 * j + tq) * 16);
        dst[1][j] = ld_stream(p1 + (4 * j + tq) * 16);
      }
    };

    int kt = warp;  // this warp's tiles: local indices warp, warp+8, ... of the piece
    if (kt < p.n) {
      int64_t r0, r1, n0 = 0, n1 = 0;
      raw_slots(p.t0 + kt, r0, r1);
      if (kt + kWarps < p.n) raw_slots(p.t0 + kt + kWarps, n0, n1);
      int64_t s0 = resolve_slot(r0, a.num_slots, a.slot_mode, err);
      int64_t s1 = resolve_slot(r1, a.num_slots, a.slot_mode, err);
      load_rows(kbase, s0, s1, kr);
      load_rows(vbase, s0, s1, vr);
      for (; kt < p.n; kt += kWarps) {
        const bool has_next = kt + kWarps < p.n;
        int64_t nn0 = 0, nn1 = 0;  // slots two tiles ahead
        if (kt + 2 * kWarps < p.n) raw_slots(p.t0 + kt + 2 * kWarps, nn0, nn1);
        // ---- S^T = K.Q^T (two accumulators halve the dependent mma chain)
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const uint4 qv = *reinterpret_cast<const uint4*>(q_s + gq * C::kQStride + 32 * j + 8 * tq);
          mma_bf16(sa, kr[0][j].x, kr[1][j].x, kr[0][j].y, kr[1][j].y, qv.x, qv.y);
          mma_bf16(sb, kr[0][j].z, kr[1][j].z, kr[0][j].w, kr[1][j].w, qv.z, qv.w);
        }
        int64_t ns0 = 0, ns1 = 0;
        if (has_next) {
          ns0 = resolve_slot(n0, a.num_slots, a.slot_mode, err);
          ns1 = resolve_slot(n1, a.num_slots, a.slot_mode, err);
          load_rows(kbase, ns0, ns1, kr);
        }
        // ---- online softmax (rows = tokens g, g+8; columns = query heads 2tq, 2tq+1)
        const int64_t tok = (int64_t)(p.t0 + kt) * kTileTok + gq;
        const bool v_lo = tok < L, v_hi = tok + 8 < L;
        float sc0 = v_lo ? (sa[0] + sb[0]) * scale_log2 : -INFINITY;
        float sc1 = v_lo ? (sa[1] + sb[1]) * scale_log2 : -INFINITY;
        float sc2 = v_hi ? (sa[2] + sb[2]) * scale_log2 : -INFINITY;
        float sc3 = v_hi ? (sa[3] + sb[3]) * scale_log2 : -INFINITY;
        float mx0 = fmaxf(sc0, sc2), mx1 = fmaxf(sc1, sc3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        const float p0 = exp2f(sc0 - mn0), p1 = exp2f(sc1 - mn1);
        const float p2 = exp2f(sc2 - mn0), p3 = exp2f(sc3 - mn1);
        l0 = l0 * al0 + p0 + p2;
        l1 = l1 * al1 + p1 + p3;
        const uint32_t pb0 = movmatrix_t(pack_bf16(p0, p1));
        const uint32_t pb1 = movmatrix_t(pack_bf16(p2, p3));
        // ---- O^T += V^T.P^T
#pragma unroll
        for (int j = 0; j < NB; ++j) {
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            float* ac = acc[j][q2];
            ac[0] *= al0;
            ac[1] *= al1;
            ac[2] *= al0;
            ac[3] *= al1;
            const uint32_t a0 = movmatrix_t(word(vr[0][j], 2 * q2));
            const uint32_t a1 = movmatrix_t(word(vr[0][j], 2 * q2 + 1));
            const uint32_t a2 = movmatrix_t(word(vr[1][j], 2 * q2));
            const uint32_t a3 = movmatrix_t(word(vr[1][j], 2 * q2 + 1));
            mma_bf16(ac, a0, a1, a2, a3, pb0, pb1);
          }
        }
        if (has_next) load_rows(vbase, ns0, ns1, vr);
        n0 = nn0;
        n1 = nn1;
      }
    }

    // ---------------- merge the eight warps of this piece ----------------
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
    __syncthreads();
    float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      M0 = fmaxf(M0, m_s[w * kHeads + 2 * tq]);
      M1 = fmaxf(M1, m_s[w * kHeads + 2 * tq + 1]);
    }
    const float f0 = m0 == -INFINITY ? 0.f : exp2f(m0 - M0);
    const float f1 = m1 == -INFINITY ? 0.f : exp2f(m1 - M1);
    float* ow = o_s + warp * kHeads * C::kOStride;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        // rows g / g+8 of A tile (j, q2) are dims phi_{2q2}(g) / phi_{2q2+1}(g)
        const int d_lo = 32 * j + 8 * (gq >> 1) + 4 * q2 + (gq & 1);
        const int d_hi = d_lo + 2;
        ow[(2 * tq) * C::kOStride + d_lo] = acc[j][q2][0] * f0;
        ow[(2 * tq + 1) * C::kOStride + d_lo] = acc[j][q2][1] * f1;
        ow[(2 * tq) * C::kOStride + d_hi] = acc[j][q2][2] * f0;
        ow[(2 * tq + 1) * C::kOStride + d_hi] = acc[j][q2][3] * f1;
      }
    }
    __syncthreads();
    const bool complete = (p.t0 == 0 && p.n == p.nt);
    const int pslot = 2 * c + (p.g_start == g0 ? 0 : 1);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
    for (int e = tid; e < G * D; e += kThreads) {
      const int hd = e / D, d = e - hd * D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w * kHeads + hd]);
      float Ls = 0.f, o = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
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
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------
// combine: the units cut by CTA range boundaries.  Combine CTA c takes the unit holding the first
// tile of decode CTA c and merges it when c is that unit's first boundary (so each cut unit is
// merged once, by one of at most nctas CTAs, with the schedule searched in shared memory); every
// CTA also writes the NaN rows of the requests without keys b = c, c + gridDim.x, ...
// ---------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) combine_kernel(tf_paged_attn_args a, Ws ws,
                                                      int nctas_launched) {
  // int64 cg[nctas+1], then w[nctas][kHeads], ml[nctas][kHeads][2], int sl[nctas], ts[B+1]
  extern __shared__ __align__(16) float csm[];
  const int B = a.batch_size, Hkv = a.num_kv_heads;
  const int G = a.num_q_heads / Hkv;
  const int tid = threadIdx.x;
  int64_t* cgs = reinterpret_cast<int64_t*>(csm);
  float* w = reinterpret_cast<float*>(cgs + nctas_launched + 1);
  float* ml = w + nctas_launched * kHeads;
  int* sl = reinterpret_cast<int*>(ml + nctas_launched * kHeads * 2);
  int* ts = sl + nctas_launched;
  for (int i = tid; i <= B; i += blockDim.x) ts[i] = ws.tile_start[i];
  __syncthreads();
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    if (ts[b + 1] != ts[b]) continue;
    // no keys: softmax over an empty row is NaN in the reference as well
    for (int e = tid; e < Hkv * G * D; e += blockDim.x) {
      const int hq = e / D, d = e - hq * D;
      out[(int64_t)b * a.out_stride_tok + (int64_t)hq * a.out_stride_head + d] = __float2bfloat16_rn(NAN);
    }
  }
  const int64_t total = (int64_t)ts[B] * Hkv;
  const int nctas = (int64_t)nctas_launched < total ? nctas_launched : (int)total;
  for (int i = tid; i <= nctas; i += blockDim.x) cgs[i] = ws.cta_g[i];
  __syncthreads();
  const int c = blockIdx.x;
  if (c == 0 || c >= nctas) return;
  const int64_t g = cgs[c];  // this CTA's boundary: the unit cut there, merged if this is its first cut
  const int b = first_req_after(ts, B, Hkv, g);
  const int nt = ts[b + 1] - ts[b];
  const int h = (int)((g - (int64_t)ts[b] * Hkv) / nt);
  const int64_t su = (int64_t)ts[b] * Hkv + (int64_t)h * nt, eu = su + nt;
  const int c0 = cta_of(cgs, nctas, su), c1 = cta_of(cgs, nctas, eu - 1);
  if (c0 == c1 || c != c0 + 1) return;  // finished inside one CTA, or merged at its first boundary
  const int np = c1 - c0 + 1;
  for (int i = tid; i < np; i += blockDim.x) {
    const int cc = c0 + i;
    const int64_t rc = cgs[cc];
    sl[i] = 2 * cc + ((su > rc ? su : rc) == rc ? 0 : 1);
  }
  // everything above reads only the plan; the decode grid's partials are complete and visible
  // after this wait (a no-op when the launch has no programmatic dependency)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  for (int e = tid; e < np * G; e += blockDim.x) {  // every piece's (max, sum) at once
    const int i = e / G, hd = e - (e / G) * G;
    ml[(i * kHeads + hd) * 2] = ws.part_ml[(sl[i] * kHeads + hd) * 2];
    ml[(i * kHeads + hd) * 2 + 1] = ws.part_ml[(sl[i] * kHeads + hd) * 2 + 1];
  }
  __syncthreads();
  if (tid < G) {
    const int hd = tid;
    float M = -INFINITY;
    for (int i = 0; i < np; ++i) M = fmaxf(M, ml[(i * kHeads + hd) * 2]);
    float L = 0.f;
    for (int i = 0; i < np; ++i) {
      const float m = ml[(i * kHeads + hd) * 2];
      const float f = m == -INFINITY ? 0.f : exp2f(m - M);
      w[i * kHeads + hd] = f;
      L += ml[(i * kHeads + hd) * 2 + 1] * f;
    }
    const float inv = 1.0f / L;
    for (int i = 0; i < np; ++i) w[i * kHeads + hd] *= inv;
  }
  // this thread's outputs e = tid + 256 k: gate values and each piece's partial sums requested
  // together (a piece at a time), then the same ordered sums as one loop per output
  constexpr int kPer = kHeads * D / 256;
  const bool gated = a.gate_mode != TF_GATE_NONE && gate != nullptr;
  __nv_bfloat16 gv[kPer];
  float o[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int e = tid + k * 256;
    o[k] = 0.f;
    if (gated && e < G * D) {
      const int hd = e / D, d = e - hd * D;
      gv[k] = gate[(int64_t)b * a.gate_stride_tok + (int64_t)(h * G + hd) * a.gate_stride_head + d];
    }
  }
  __syncthreads();
  // up to four pieces' partial sums requested together, then added in piece order
  constexpr int kBatch = 4;
  for (int i0 = 0; i0 < np; i0 += kBatch) {
    float po[kBatch][kPer];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (i0 + j >= np) break;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int e = tid + k * 256;
        if (e < G * D)
          po[j][k] = ws.part_o[((int64_t)sl[i0 + j] * kHeads + e / D) * D + (e - (e / D) * D)];
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (i0 + j >= np) break;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int e = tid + k * 256;
        if (e < G * D) o[k] = fmaf(w[(i0 + j) * kHeads + e / D], po[j][k], o[k]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int e = tid + k * 256;
    if (e >= G * D) break;
    const int hd = e / D, d = e - hd * D;
    const int hq = h * G + hd;
    float r = round_to<__nv_bfloat16>(o[k]);
    if (gated) r = apply_gate<__nv_bfloat16>(r, to_f(gv[k]), a.gate_mode);
    out[(int64_t)b * a.out_stride_tok + (int64_t)hq * a.out_stride_head + d] = __float2bfloat16_rn(r);
  }
}

template <int D>
static cudaError_t launch_d(const tf_paged_attn_args& a, void* wsp, int nctas, cudaStream_t s) {
  Ws ws = carve(wsp, a.batch_size, nctas, D);
  // a unit spans at most every CTA: the combine holds the CTA boundaries [nctas+1], weights
  // [nctas][kHeads], (max, sum) [nctas][kHeads][2] and slot ids [nctas], then the schedule
  // tile_start[B+1]; checked before the first launch so that a batch it cannot hold leaves nothing
  // enqueued
  const size_t csmem = (size_t)(nctas + 1) * 8 + (size_t)nctas * (3 * kHeads * 4 + 4) +
                       (size_t)(a.batch_size + 1) * 4;
  if (nctas > kPlanMaxCtas) return cudaErrorInvalidValue;
  if (csmem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(decode_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Cfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(combine_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem);
  if (e != cudaSuccess) return e;
  plan_kernel<<<1, kPlanThreads, 0, s>>>(a.seq_lens, a.batch_size, a.r2t_cols, a.num_kv_heads, nctas,
                                         PieceCost<D>::v, ws);
  // the decode CTAs are scheduled while the plan runs and wait for it before their first read
  cudaLaunchAttribute dep[1];
  dep[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  dep[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t dcfg = {};
  dcfg.gridDim = dim3((unsigned)nctas);
  dcfg.blockDim = dim3(kThreads);
  dcfg.dynamicSmemBytes = Cfg<D>::kSmem;
  dcfg.stream = s;
  dcfg.attrs = dep;
  dcfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&dcfg, decode_kernel<D>, a, ws, nctas);
  if (e != cudaSuccess) return e;
  // programmatic dependent launch: the combine's CTAs are scheduled as the decode's CTAs exit and
  // do their schedule search while the last decode CTAs still run
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nctas);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = csmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, combine_kernel<D>, a, ws, nctas);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace dec

bool paged_decode_mma_supported(const tf_paged_attn_args& a) {
  if (a.dtype != TF_DTYPE_BF16) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  const int G = a.num_q_heads / a.num_kv_heads;
  if (G < 1 || G > dec::kHeads) return false;
  if (a.batch_size > kDecodeMmaMaxBatch) return false;
  auto al = [](const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
  if (!al(a.k_buffer, 16) || !al(a.v_buffer, 16)) return false;
  if ((a.kv_stride_slot * 2) % 16 != 0 || (a.kv_stride_head * 2) % 16 != 0) return false;
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

// ---------------------------------------------------------------------------------------------
// Allocation-free variant (tf_paged_decode_attn_noalloc).
//
// Some callers cannot allocate device memory themselves: a host runtime that binds this C ABI
// through a plain FFI and has no CUDA allocator of its own, or a serving process whose device
// memory is all handed to its own pool at start-up.  For them the decode's scratch (schedule and
// split partials) lives in this fixed file-scope array instead of a caller workspace.  Every GPU
// that loads the library holds these kNoAllocScratchBytes until the process exits; all calls on a
// device share the one array and it keeps the last call's contents, so calls whose kernels overlap
// on that GPU (other streams, other threads) race on it and must be serialised by the caller.
// ---------------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kScratchMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kScratchMaxDevices] = {};
}  // namespace

// Device address of g_decode_scratch on the stream's device.  In host code the array's name is a
// host-side stand-in, never a device address, so it is resolved once per device (with that device
// current) by cudaGetSymbolAddress.  Outside capture the C ABI has made the stream's device
// current.  While `s` is being captured the stream's device cannot be queried without breaking the
// capture, so the capturing thread's current device is taken (a captured stream must belong to it)
// and the address must already be known: the first call on a device has to come before any
// capture, and a capture that would need the lookup is refused instead of resolving it mid-capture.
static cudaError_t decode_scratch_ptr(cudaStream_t s, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kScratchMaxDevices) return cudaErrorInvalidDevice;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(s, &cap);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    if (cap != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

cudaError_t launch_paged_decode_mma_noalloc(const tf_paged_attn_args& a, int num_sms,
                                            cudaStream_t s) {
  void* ws = nullptr;
  cudaError_t e = decode_scratch_ptr(s, &ws);
  if (e != cudaSuccess) return e;
  // the status word keeps the previous call's error code: start every call from zero
  e = cudaMemsetAsync(ws, 0, 256, s);
  if (e != cudaSuccess) return e;
  return launch_paged_decode_mma(a, ws, kNoAllocScratchBytes, num_sms, s);
}

}  // namespace tf
