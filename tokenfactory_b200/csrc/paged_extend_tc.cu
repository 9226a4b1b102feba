// a3 + a4: paged GQA extend / prefill attention over a radix-cached prefix on the 5th-generation
// tensor cores (qwen3_8/full_attention.py:179-213 and :244-283, output gate :157-158).
//
// One CTA owns 128 query rows: 128/G consecutive query tokens of one request times the G query
// heads that share kv head h (GQA packed into M), and walks the visible keys in tiles of 64 token
// rows gathered through req_to_token.  The CTA is warp-specialised:
//   warps 0-3  softmax: thread r owns row r (TMEM lane r).  Reads S_j from TMEM, applies the causal
//              mask and an online max/sum with a lazy rescale (O is rescaled in TMEM only when a
//              row's max grows by more than 2^8), writes P_j as bf16 into TMEM, then runs the
//              epilogue (O / l, output gate, bf16 store).
//   warps 4-7  producers: load Q once, then gather K and V rows (one 16-byte cp.async per lane,
//              whole rows per warp instruction) into a ring of SWIZZLE_128B slots; each slot holds
//              the K or the V half of a key tile and is filled in the order the MMAs consume it
//              (K0 K1 V0 K2 V1 K3 ...).  Completion is tracked by cp.async.mbarrier.arrive.
//   warp 8     one thread issues the tcgen05.mma chain: S_0, S_1, then per tile PV_j followed by
//              S_{j+2}, so the tensor core computes while the softmax of tile j+1 runs.
//                S = Q.K^T    M128 N64 K16 x D/16, A and B from shared memory
//                O += P.V     M128 N=D K16 x 4, A (P) from TMEM, B (V) MN-major in shared memory
// TMEM holds two S buffers, O, and two P buffers, so no MMA overwrites an operand that an
// earlier MMA still reads.  Every wait is bounded; a wait that gives up raises a CTA-wide abort
// flag, the other roles leave their loops, and the kernel records TF_KERR_TIMEOUT.  Rows past the
// end of the request and keys outside a row's causal window are masked; query i of request b
// sees keys j <= seq_len - extend_len + i.
#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace tf {
namespace ext {

constexpr int kRows = 128;
constexpr int kBN = 64;
constexpr int kSoftmaxWarps = 4;
constexpr int kProducerWarps = 4;
constexpr int kMmaWarp = kSoftmaxWarps + kProducerWarps;
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr int kProducerThreads = kProducerWarps * 32;
constexpr int kRowsPerProducer = kBN / kProducerWarps;  // key rows of a tile per producer warp
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;

template <int D>
struct Cfg {
  static constexpr int kKB = D / 64;             // 64-element blocks of a row
  static constexpr int kQBlock = kRows * 128;    // one 64-dim block of Q
  static constexpr int kKVBlock = kBN * 128;     // one 64-dim block of a K or V tile
  static constexpr int kQBytes = kKB * kQBlock;
  static constexpr int kSlotBytes = kKB * kKVBlock;
  static constexpr int kSlots = D == 256 ? 5 : (D == 128 ? 10 : 8);
  static constexpr int kOffRing = kQBytes;
  static constexpr int kOffBars = kOffRing + kSlots * kSlotBytes;
  // barriers: full[kSlots], empty[kSlots], s_full[2], p_full[2], o_done, q_full, fin
  static constexpr int kNumBars = 2 * kSlots + 7;
  static constexpr int kOffWords = kOffBars + 8 * kNumBars;   // tmem holder, abort, q0 (int64)
  static constexpr int kOffSlotIds = kOffWords + 16;          // int64 [2][kBN]
  static constexpr int kSmem = kOffSlotIds + 2 * kBN * 8 + 1024;  // + slack to align the base
  static constexpr int kColS = 0;                 // S buffers at [0,64) and [64,128)
  static constexpr int kColO = 2 * kBN;           // O: D columns
  static constexpr int kColP = kColO + D;         // P buffers: 32 columns each (bf16 pairs)
  static constexpr int kTmemCols = kColP + kBN <= 256 ? 256 : 512;
  static_assert(D % 64 == 0, "head_dim multiple of 64");
  static_assert(kSmem <= 232448, "shared memory per CTA");
  static_assert(kOffSlotIds % 8 == 0, "slot id alignment");
};

// Bounded mbarrier wait that also gives up when another role raised the abort flag.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kSpinLimitNs) {
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// max of 64 scores as a tree of three-input maxima (depth 4 instead of a 64-long chain)
__device__ __forceinline__ float max_of_64(const float (&s)[2][32]) {
  float t[22];
#pragma unroll
  for (int i = 0; i < 21; ++i) {
    const int k = 3 * i;
    t[i] = max3(s[k >> 5][k & 31], s[(k + 1) >> 5][(k + 1) & 31], s[(k + 2) >> 5][(k + 2) & 31]);
  }
  t[21] = s[1][31];
  float u[8];
#pragma unroll
  for (int i = 0; i < 7; ++i) u[i] = max3(t[3 * i], t[3 * i + 1], t[3 * i + 2]);
  u[7] = t[21];
  return fmaxf(max3(u[0], u[1], u[2]), max3(u[3], u[4], max3(u[5], u[6], u[7])));
}
// 2^x with the hardware approximation (flush-to-zero): x = -inf gives +0
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    extend_kernel(tf_paged_attn_args a, int tiles_per_req) {
  using C = Cfg<D>;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw_base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + C::kOffBars);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kSlots;
  uint64_t* s_full = bars + 2 * C::kSlots;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* q_full = o_done + 1;
  uint64_t* fin = q_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sbase + C::kOffWords);
  volatile int* abort = reinterpret_cast<volatile int*>(sbase + C::kOffWords + 4);
  int64_t* s_q0 = reinterpret_cast<int64_t*>(sbase + C::kOffWords + 8);
  int64_t* slot_ids = reinterpret_cast<int64_t*>(sbase + C::kOffSlotIds);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hkv = a.num_kv_heads, G = a.num_q_heads / Hkv;
  const int TQ = kRows / G;  // query tokens per CTA
  const int b = blockIdx.x / tiles_per_req;
  const int qt = tiles_per_req - 1 - (blockIdx.x - b * tiles_per_req);  // longest tiles first
  const int h = blockIdx.y;
  const int64_t E = a.extend_lens ? a.extend_lens[b] : 1;
  const int64_t tile_start = (int64_t)qt * TQ;
  if (tile_start >= E) return;
  const int64_t L = a.seq_lens[b];
  if (L > a.r2t_cols || L < E) {  // a length the req_to_token table cannot hold
    if (tid == 0) record_err(a.err, TF_KERR_SLOT_RANGE);
    return;
  }
  const int64_t P = L - E;
  const int n_tok = (int)(E - tile_start < TQ ? E - tile_start : TQ);
  const int64_t kv_end = P + tile_start + n_tok;  // keys [0, kv_end) are visible to some row
  const int ntiles = (int)((kv_end + kBN - 1) / kBN);

  if (warp == 0) {  // token offset of request b: exclusive prefix of extend_lens
    int64_t acc = 0;
    for (int i = lane; i < b; i += 32) acc += a.extend_lens ? a.extend_lens[i] : 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) *s_q0 = acc;
  }
  if (tid == 0) {
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&full[i], kProducerThreads);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftmaxWarps);
    }
    mbar_init(o_done, 1);
    mbar_init(q_full, kProducerThreads);
    mbar_init(fin, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tc::tmem_alloc(tmem_holder, C::kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const int64_t q0 = *s_q0 + tile_start;

  if (warp >= kSoftmaxWarps && warp < kMmaWarp) {
    // ======================= producers =======================
    const int pw = warp - kSoftmaxWarps;
    constexpr int CPR = D / 8;          // 16-byte chunks per row
    constexpr int RPI = 32 / CPR;       // rows per warp instruction
    const int sub = lane / CPR, ch = lane - (lane / CPR) * CPR;
    // Q: 128 rows, pw owns rows [32 pw, 32 pw + 32); rows past the request end are zero
    {
      const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q);
#pragma unroll 4
      for (int i = 0; i < 32; i += RPI) {
        const int r = pw * 32 + i + sub;
        const int ti = r / G, g = r - (r / G) * G;
        const bool v = ti < n_tok;
        const __nv_bfloat16* src =
            v ? q + (q0 + ti) * a.q_stride_tok + (int64_t)(h * G + g) * a.q_stride_head + ch * 8
              : q;
        const uint32_t dst = base + (ch >> 3) * C::kQBlock + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
        cp_async16_zfill(dst, src, v ? 16u : 0u);
      }
      cp_async_arrive_noinc(q_full);
    }
    int64_t row = a.req_pool_indices[b];
    if (row < 0 || row >= a.r2t_rows) {
      if (tid == kSoftmaxWarps * 32) record_err(a.err, TF_KERR_REQ_RANGE);
      row = 0;
    }
    const int64_t* r2t = a.req_to_token + row * a.r2t_stride;
    const char* kbuf = (const char*)a.k_buffer + (int64_t)h * a.kv_stride_head * 2;
    const char* vbuf = (const char*)a.v_buffer + (int64_t)h * a.kv_stride_head * 2;
    const int64_t sstride = a.kv_stride_slot * 2;
    const int seg = pw * kRowsPerProducer;
    auto raw_of = [&](int tile) -> int64_t {  // lanes < kRowsPerProducer: key of this lane's row
      int64_t key = (int64_t)tile * kBN + seg + lane;
      if (key >= kv_end) key = (int64_t)tile * kBN;  // past the window: repeat the tile's first key
      return r2t[key];
    };
    // raw req_to_token entries of the next kPrefetch K tiles: this load returns behind the
    // tile gathers already in flight, so it is issued several tiles ahead of its use
    constexpr int kPrefetch = 4;
    int64_t raw_q[kPrefetch];
#pragma unroll
    for (int i = 0; i < kPrefetch; ++i) raw_q[i] = (lane < kRowsPerProducer && i < ntiles) ? raw_of(i) : 0;
    int slot = 0;
    uint32_t phase = 0;
    bool ok = true;
    auto produce = [&](int tile, bool isv) {
      const bool got = wait_bar(&empty[slot], phase ^ 1u, abort);
      ok = __all_sync(0xffffffffu, got);
      if (!ok) return;
      int64_t* ids = slot_ids + (tile & 1) * kBN + seg;
      if (!isv) {
        const int64_t raw = raw_q[0];
#pragma unroll
        for (int i = 0; i + 1 < kPrefetch; ++i) raw_q[i] = raw_q[i + 1];
        raw_q[kPrefetch - 1] =
            (tile + kPrefetch < ntiles && lane < kRowsPerProducer) ? raw_of(tile + kPrefetch) : 0;
        if (lane < kRowsPerProducer) ids[lane] = resolve_slot(raw, a.num_slots, a.slot_mode, a.err);
        __syncwarp();
      }
      const char* src0 = (isv ? vbuf : kbuf) + ch * 16;
      const uint32_t dst0 = base + C::kOffRing + slot * C::kSlotBytes + (ch >> 3) * C::kKVBlock;
#pragma unroll
      for (int i = 0; i < kRowsPerProducer; i += RPI) {
        const int r = seg + i + sub;  // key row in the tile
        const int64_t sl = ids[i + sub];
        cp_async16(dst0 + r * 128 + (((ch & 7) ^ (r & 7)) << 4), src0 + sl * sstride);
      }
      cp_async_arrive_noinc(&full[slot]);
      if (++slot == C::kSlots) { slot = 0; phase ^= 1u; }
    };
    produce(0, false);
    if (ok && ntiles > 1) produce(1, false);
    for (int j = 0; ok && j < ntiles; ++j) {
      produce(j, true);
      if (ok && j + 2 < ntiles) produce(j + 2, false);
    }
    cp_async_wait_all();
  } else if (warp == kMmaWarp) {
    // ======================= MMA issue (one thread) =======================
    if (lane == 0) {
      constexpr uint32_t kIdS = tc::idesc_bf16(kRows, kBN, false, false);
      constexpr uint32_t kIdO = tc::idesc_bf16(kRows, D, false, true);
      bool ok = wait_bar(q_full, 0, abort);
      tc::fence_proxy_async_smem();
      int slot = 0;
      uint32_t phase = 0;
      auto take = [&]() -> uint32_t {  // wait for the next ring slot; returns its address
        ok = ok && wait_bar(&full[slot], phase, abort);
        tc::fence_proxy_async_smem();
        return base + C::kOffRing + slot * C::kSlotBytes;
      };
      auto release = [&]() {
        tc::commit(&empty[slot]);
        if (++slot == C::kSlots) { slot = 0; phase ^= 1u; }
      };
      auto issue_s = [&](int t) {
        const uint32_t kb = take();
        if (!ok) return;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::sw128_desc(base + (kk >> 2) * C::kQBlock + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sw128_desc(kb + (kk >> 2) * C::kKVBlock + (kk & 3) * 32, 16, 1024);
          tc::mma_bf16(tmem + C::kColS + (t & 1) * kBN, ad, bd, kIdS, kk > 0);
        }
        tc::commit(&s_full[t & 1]);
        release();
      };
      auto issue_pv = [&](int t) {
        ok = ok && wait_bar(&p_full[t & 1], (t >> 1) & 1, abort);
        tc::fence_after_sync();
        const uint32_t vb = take();
        if (!ok) return;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bd = tc::sw128_desc(vb + kk * 2048, C::kKVBlock, 1024);
          tc::mma_bf16_ts(tmem + C::kColO, tmem + C::kColP + (t & 1) * (kBN / 2) + kk * 8, bd, kIdO,
                          t > 0 || kk > 0);
        }
        tc::commit(o_done);
        release();
      };
      if (ok) issue_s(0);
      if (ok && ntiles > 1) issue_s(1);
      for (int j = 0; ok && j < ntiles; ++j) {
        issue_pv(j);
        if (ok && j + 2 < ntiles) issue_s(j + 2);
      }
      // every MMA issued above has completed before TMEM is read for the last time or released
      tc::commit(fin);
      // waited for also after an abort (bounded): no MMA may be in flight when TMEM is released
      if (!mbar_wait(fin, 0)) *abort = 1;
    }
    __syncwarp();
  } else {
    // ======================= softmax + epilogue (thread r = row r) =======================
    const float c2 = a.scale * kLog2e;
    const int r = tid;
    const int ri = r / G, rg = r - (r / G) * G;
    const bool row_valid = ri < n_tok;
    const int64_t klim = P + tile_start + ri + 1;  // keys [0, klim) visible to this row
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int bi = j & 1;
      ok = __all_sync(0xffffffffu, wait_bar(&s_full[bi], (j >> 1) & 1, abort));
      if (!ok) break;
      tc::fence_after_sync();
      float s[2][32];
      tc::ld32(tmem + lane_base + C::kColS + bi * kBN, s[0]);
      tc::ld32(tmem + lane_base + C::kColS + bi * kBN + 32, s[1]);
      tc::wait_ld();
      const int64_t key0 = (int64_t)j * kBN;
      // raw scores: masked keys become -inf, the max is taken on raw scores (c2 > 0; the host
      // routes c2 <= 0 elsewhere) and the scale is folded into the exponent's FFMA
      if (!(row_valid && key0 + kBN <= klim)) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (!(row_valid && key0 + hh * 32 + k < klim)) s[hh][k] = -INFINITY;
      }
      const float tmax = max_of_64(s) * c2;
      const bool need = tmax > m_used + kRescaleLog2 || (m_used == -INFINITY && tmax > -INFINITY);
      const float m_new = need ? tmax : m_used;
      const float alpha = need ? (m_used == -INFINITY ? 0.f : exp2f(m_used - m_new)) : 1.f;
      m_used = m_new;
      l_sum *= alpha;
      if (j > 0 && __any_sync(0xffffffffu, need)) {  // rescale this warp's O rows (PV_{j-1} done)
        ok = __all_sync(0xffffffffu, wait_bar(o_done, (j - 1) & 1, abort));
        if (!ok) break;
        tc::fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          float o[32];
          tc::ld32(tmem + lane_base + C::kColO + cc * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] *= alpha;
          tc::st32(tmem + lane_base + C::kColO + cc * 32, o);
        }
      }
      // P_j in bf16 -> TMEM (32 columns of bf16 pairs)
      const float nmu = m_used == -INFINITY ? 0.f : -m_used;
      float pk[32];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k2 = 0; k2 < 32; ++k2) {
        const float p0 = ex2_ftz(fmaf(s[k2 >> 4][(2 * k2) & 31], c2, nmu));
        const float p1 = ex2_ftz(fmaf(s[k2 >> 4][(2 * k2 + 1) & 31], c2, nmu));
        ls[k2 & 3] += p0 + p1;
        __nv_bfloat162 pv = __floats2bfloat162_rn(p0, p1);
        pk[k2] = __uint_as_float(*reinterpret_cast<uint32_t*>(&pv));
      }
      l_sum += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tc::st32(tmem + lane_base + C::kColP + bi * (kBN / 2), pk);
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[bi]);
    }
    // ---- epilogue: O / l, output gate, bf16
    // fin (one phase, committed after the last PV) rather than o_done: o_done can still be two
    // phases short here, since PV_{n-2} is issued after S_{n-1}
    if (ok) ok = __all_sync(0xffffffffu, wait_bar(fin, 0, abort));
    if (ok) {
      tc::fence_after_sync();
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
      const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
      const bool gated = a.gate_mode != TF_GATE_NONE && gate != nullptr;
      const bool vec = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(gate)) & 15) == 0 &&
                       (a.out_stride_tok | a.out_stride_head | a.gate_stride_tok | a.gate_stride_head) % 8 == 0;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const int64_t t = q0 + ri;
      const int hq = h * G + rg;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        tc::ld32(tmem + lane_base + C::kColO + cc * 32, o);
        tc::wait_ld();
        if (!row_valid) continue;
        __nv_bfloat16* op = out + t * a.out_stride_tok + (int64_t)hq * a.out_stride_head + cc * 32;
        const __nv_bfloat16* gp =
            gated ? gate + t * a.gate_stride_tok + (int64_t)hq * a.gate_stride_head + cc * 32 : nullptr;
        if (vec) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint4 gw = make_uint4(0, 0, 0, 0);
            if (gated) gw = *reinterpret_cast<const uint4*>(gp + c8 * 8);
            const __nv_bfloat16* gv = reinterpret_cast<const __nv_bfloat16*>(&gw);
            uint4 ow;
            __nv_bfloat16* ov = reinterpret_cast<__nv_bfloat16*>(&ow);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              float v = round_to<__nv_bfloat16>(l_sum > 0.f ? o[c8 * 8 + k] * inv : NAN);
              if (gated) v = apply_gate<__nv_bfloat16>(v, to_f(gv[k]), a.gate_mode);
              ov[k] = __float2bfloat16_rn(v);
            }
            *reinterpret_cast<uint4*>(op + c8 * 8) = ow;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            float v = round_to<__nv_bfloat16>(l_sum > 0.f ? o[k] * inv : NAN);
            if (gated) v = apply_gate<__nv_bfloat16>(v, to_f(gp[k]), a.gate_mode);
            op[k] = __float2bfloat16_rn(v);
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && *abort) record_err(a.err, TF_KERR_TIMEOUT);
  tc::fence_after_sync();
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, C::kTmemCols);
}

template <int D>
static cudaError_t launch_d(const tf_paged_attn_args& a, cudaStream_t s) {
  const int G = a.num_q_heads / a.num_kv_heads;
  const int TQ = kRows / G;
  const int tiles = (a.max_extend_len + TQ - 1) / TQ;
  cudaError_t e = cudaFuncSetAttribute(extend_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)(a.batch_size * tiles), (unsigned)a.num_kv_heads);
  extend_kernel<D><<<grid, kThreads, Cfg<D>::kSmem, s>>>(a, tiles);
  return cudaGetLastError();
}


// =============================================================================================
// Pair kernel (head_dim 128 / 256): two CTAs of a cluster on an SM pair run one M=256 tile with
// tcgen05.mma.cta_group::2.  CTA r holds query rows [128 r, 128 r + 128) of the pair tile, and of
// every key tile only keys [32 r, 32 r + 32) of K and dims [r D/2, (r+1) D/2) of V: the MMA reads
// the B operand from both CTAs' shared memory, so each SM gathers half of the K/V bytes.
//   rank 0, warp 8: issues every MMA of the pair; commits arrive on both CTAs' barriers
//   rank 1, warp 8: relays "this CTA's half of slot s has landed" to rank 0's full barrier
//   warps 0-3 of each CTA: softmax + epilogue of its own 128 rows (own TMEM)
//   warps 4-7 of each CTA: gather its halves into its own ring
// =============================================================================================
namespace pair {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// Arrive on the peer CTA's barrier.  CTA-scope release, the arrive form CUTLASS's cluster barriers
// use: what the waiter goes on to read (this CTA's shared memory through the pair MMA, this CTA's
// TMEM) is complete behind the tcgen05 / proxy fences that precede every call.  A cluster-scope
// release also drains this thread's earlier remote arrives first, which serialised the per-slot
// relay: config 4 ran at 919 TFLOP/s with it against 974 without.
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void remote_store(uint32_t cluster_addr, int v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire; on timeout raises the abort flag of both CTAs.
__device__ __forceinline__ bool wait_c(uint64_t* bar, uint32_t parity, volatile int* abort,
                                       uint32_t peer_abort) {
  const uint32_t addr = smem_u32(bar);
  if (try_wait_cluster(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (try_wait_cluster(addr, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kSpinLimitNs) {
        *abort = 1;
        remote_store(peer_abort, 1);
        return false;
      }
    }
  }
}
// Same with the default (CTA-scope) acquire, for the many threads that poll barriers completed by
// tcgen05.commit or by this CTA's own cp.async: what they read next is TMEM or this CTA's shared
// memory behind tcgen05 / proxy fences, so no cluster-scope acquire is needed on their hot path.
// Bounded wait that does not stop for the abort flag: the issuing thread drains the pair's MMAs
// before either CTA releases TMEM, also after an abort.
__device__ __forceinline__ bool drain_c(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (try_wait_cluster(addr, parity)) return true;
    if ((it & 63u) == 63u && global_ns() - t0 > kSpinLimitNs) return false;
  }
}
__device__ __forceinline__ bool wait_l(uint64_t* bar, uint32_t parity, volatile int* abort,
                                       uint32_t peer_abort, unsigned backoff_ns = 0) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (backoff_ns) __nanosleep(backoff_ns);
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kSpinLimitNs) {
        *abort = 1;
        remote_store(peer_abort, 1);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void mma2_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc ? 1u : 0u)
      : "memory");
}
__device__ __forceinline__ void mma2_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc ? 1u : 0u)
      : "memory");
}
// arrive once on the barrier at this offset in both CTAs when all prior MMAs have completed
__device__ __forceinline__ void commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)), "h"((uint16_t)3)
      : "memory");
}

constexpr int kPBN = 128;                       // keys per tile: S = Q.K^T is M256 x N128
constexpr int kSmWarps = 8;                    // two warps per 32-row group: key columns 0-31 / 32-63
constexpr int kPrWarp0 = kSmWarps;             // producers: warps 8-11
constexpr int kIssueWarp = kSmWarps + kProducerWarps;  // MMA issue (rank 0) / slot relay (rank 1)
constexpr int kFwdWarp = kIssueWarp + 1;               // rank 1: forwards "P written" to rank 0
constexpr int kPairThreads = (kFwdWarp + 1) * 32;

// Output-gate activation for the epilogue: sigmoid as a hardware reciprocal of 1 + e^-x (within a
// few fp32 ulp of the IEEE quotient, far below the bf16 rounding that follows); silu = x sigmoid(x).
__device__ __forceinline__ float act_fast(float x, int mode) {
  float sg;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(sg) : "f"(1.0f + __expf(-x)));
  return mode == TF_GATE_SILU ? x * sg : sg;
}

// gate and output rows can be moved in 16-byte pieces
__device__ __forceinline__ bool gate_vec(const tf_paged_attn_args& a) {
  return ((reinterpret_cast<uintptr_t>(a.out) | reinterpret_cast<uintptr_t>(a.gate)) & 15) == 0 &&
         (a.out_stride_tok | a.out_stride_head | a.gate_stride_tok | a.gate_stride_head) % 8 == 0;
}

// p = 2^(s c2 - m) for 32 scores, packed as 16 bf16 pairs; returns the sum of the fp32 p
__device__ __forceinline__ float exp_pack(const float (&sh)[32], float c2, float nmu, float (&pk)[16]) {
  float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int k2 = 0; k2 < 16; ++k2) {
    const float p0 = ex2_ftz(fmaf(sh[2 * k2], c2, nmu));
    const float p1 = ex2_ftz(fmaf(sh[2 * k2 + 1], c2, nmu));
    ls[k2 & 3] += p0 + p1;
    __nv_bfloat162 pv = __floats2bfloat162_rn(p0, p1);
    pk[k2] = __uint_as_float(*reinterpret_cast<uint32_t*>(&pv));
  }
  return (ls[0] + ls[1]) + (ls[2] + ls[3]);
}

template <int D>
struct Cfg {
  static constexpr int kKB = D / 64;
  static constexpr int kQBlock = kRows * 128;       // one 64-dim block of this CTA's Q rows
  static constexpr int kQBytes = kKB * kQBlock;
  static constexpr int kKBlk = (kPBN / 2) * 128;    // K half: 64 keys x 128 B per 64-dim block
  static constexpr int kVBlk = kPBN * 128;          // V half: 128 keys x 128 B per 64-dim block
  static constexpr int kSlotBytes = kKB * kKBlk;    // == (kKB / 2) * kVBlk
  static constexpr int kSlots = D == 256 ? 4 : 8;
  static constexpr int kOffRing = kQBytes;
  static constexpr int kOffBars = kOffRing + kSlots * kSlotBytes;
  static constexpr int kNumBars = 2 * kSlots + 8;   // full, empty, s_full[2], p_full[2], o_done, q_full, fin, q_dead
  static constexpr int kOffWords = kOffBars + 8 * kNumBars;
  static constexpr int kOffIds = kOffWords + 16;    // int64 [2][kProducerWarps][32]
  static constexpr int kOffPmax = kOffIds + 2 * kProducerWarps * 32 * 8;  // float [2][2][kRows]
  static constexpr int kSmem = kOffPmax + 2 * 2 * kRows * 4 + 1024;
  static constexpr int kColS = 0;                   // two S buffers of kPBN columns; P_j over S_j
  static constexpr int kColO = 2 * kPBN;
  static constexpr int kTmemCols = 512;
  static_assert(D == 128 || D == 256, "pair kernel head dims");
  static_assert(kSlotBytes == (kKB / 2) * kVBlk, "K and V halves share the slot size");
  static_assert(kSmem <= 232448, "shared memory per CTA");
  static_assert(kColO + D <= kTmemCols, "TMEM columns");
  static_assert(kRows * D * 2 + 2 * kRows * 4 <= kSlots * kSlotBytes, "epilogue stage fits the ring");
};

template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    extend_pair_kernel(tf_paged_attn_args a, int pairs_per_req) {
  using C = Cfg<D>;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw_base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + C::kOffBars);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kSlots;
  uint64_t* s_full = bars + 2 * C::kSlots;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* q_full = o_done + 1;
  uint64_t* fin = q_full + 1;
  uint64_t* q_dead = fin + 1;  // the last S MMA has completed: Q's shared memory is free
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sbase + C::kOffWords);
  volatile int* abort = reinterpret_cast<volatile int*>(sbase + C::kOffWords + 4);
  int64_t* s_q0 = reinterpret_cast<int64_t*>(sbase + C::kOffWords + 8);
  int64_t* ids_all = reinterpret_cast<int64_t*>(sbase + C::kOffIds);
  float* pmax = reinterpret_cast<float*>(sbase + C::kOffPmax);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t peer = rank ^ 1u;
  const uint32_t peer_abort = peer_addr(smem_u32((const void*)abort), peer);
  const int Hkv = a.num_kv_heads, G = a.num_q_heads / Hkv;
  const int TQ = kRows / G;  // query tokens per CTA
  const int pidx = blockIdx.x >> 1;
  const int b = pidx / pairs_per_req;
  const int qp = pairs_per_req - 1 - (pidx - b * pairs_per_req);  // longest pair tiles first
  const int h = blockIdx.y;
  const int64_t E = a.extend_lens ? a.extend_lens[b] : 1;
  const int64_t pair_start = (int64_t)qp * 2 * TQ;
  if (pair_start >= E) return;  // both CTAs of the pair leave here, before any cluster barrier
  const int64_t L = a.seq_lens[b];
  if (L > a.r2t_cols || L < E) {
    if (tid == 0 && rank == 0) record_err(a.err, TF_KERR_SLOT_RANGE);
    return;
  }
  const int64_t P = L - E;
  const int64_t cta_start = pair_start + (int64_t)rank * TQ;  // first token of this CTA's rows
  const int n_tok = (int)(E - cta_start <= 0 ? 0 : (E - cta_start < TQ ? E - cta_start : TQ));
  const int64_t pair_end = E - pair_start < 2 * TQ ? E : pair_start + 2 * TQ;
  const int64_t kv_end = P + pair_end;  // keys [0, kv_end) are visible to some row of the pair
  const int ntiles = (int)((kv_end + kPBN - 1) / kPBN);

  if (warp == 0) {
    int64_t acc = 0;
    for (int i = lane; i < b; i += 32) acc += a.extend_lens ? a.extend_lens[i] : 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) *s_q0 = acc;
  }
  if (tid == 0) {
    const uint32_t in_count = rank == 0 ? kProducerThreads + 1 : kProducerThreads;
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&full[i], in_count);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], rank == 0 ? kSmWarps + 1 : kSmWarps);
    }
    mbar_init(o_done, 1);
    mbar_init(q_full, in_count);
    mbar_init(fin, 1);
    mbar_init(q_dead, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // producers: the slot-id chain of the first key tiles (the request's req_to_token row, then its
  // entries) is requested before the set-up barrier, so that its two round trips overlap the set-up
  // and the copies of Q.  Lane l < 16 takes key 64 rank + 16 pw + l (this CTA's K rows and V rows),
  // lane l >= 16 key 64 (1 - rank) + 16 pw + l - 16 (V rows only): a warp's V rows include its K rows
  constexpr int kPrefetch = 4;
  int64_t raw_q[kPrefetch] = {0, 0, 0, 0};
  const int64_t* r2t = a.req_to_token;
  int my_key = 0;
  if (warp >= kPrWarp0 && warp < kIssueWarp) {
    const int pw = warp - kPrWarp0;
    int64_t row = a.req_pool_indices[b];
    if (row < 0 || row >= a.r2t_rows) {
      if (tid == kPrWarp0 * 32 && rank == 0) record_err(a.err, TF_KERR_REQ_RANGE);
      row = 0;
    }
    r2t = a.req_to_token + row * a.r2t_stride;
    my_key = lane < 16 ? 64 * (int)rank + 16 * pw + lane : 64 * (1 - (int)rank) + 16 * pw + lane - 16;
#pragma unroll
    for (int i = 0; i < kPrefetch; ++i) {
      int64_t key = (int64_t)i * kPBN + my_key;
      if (key >= kv_end) key = (int64_t)i * kPBN;  // past the window: repeat the tile's first key
      if (i < ntiles) raw_q[i] = r2t[key];
    }
  }
  if (warp == kIssueWarp) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)), "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc::fence_before_sync();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const int64_t q0 = *s_q0 + cta_start;

  if (warp >= kPrWarp0 && warp < kIssueWarp) {
    // ======================= producers: this CTA's halves =======================
    const int pw = warp - kPrWarp0;
    {  // Q: this CTA's 128 rows
      constexpr int CPR = D / 8, RPI = 32 / CPR;
      const int sub = lane / CPR, ch = lane - (lane / CPR) * CPR;
      const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q);
#pragma unroll 4
      for (int i = 0; i < 32; i += RPI) {
        const int r = pw * 32 + i + sub;
        const int ti = r / G, g = r - (r / G) * G;
        const bool v = ti < n_tok;
        const __nv_bfloat16* src =
            v ? q + (q0 + ti) * a.q_stride_tok + (int64_t)(h * G + g) * a.q_stride_head + ch * 8 : q;
        cp_async16_zfill(base + (ch >> 3) * C::kQBlock + r * 128 + (((ch & 7) ^ (r & 7)) << 4), src,
                         v ? 16u : 0u);
      }
      cp_async_arrive_noinc(q_full);
    }
    const char* kbuf = (const char*)a.k_buffer + (int64_t)h * a.kv_stride_head * 2;
    const char* vbuf = (const char*)a.v_buffer + (int64_t)h * a.kv_stride_head * 2 + rank * D;
    const int64_t sstride = a.kv_stride_slot * 2;
    auto raw_of = [&](int tile) -> int64_t {
      int64_t key = (int64_t)tile * kPBN + my_key;
      if (key >= kv_end) key = (int64_t)tile * kPBN;  // past the window: repeat the tile's first key
      return r2t[key];
    };
    int slot = 0;
    uint32_t phase = 0;
    bool ok = true;
    auto produce = [&](int tile, bool isv) {
      // producers run far ahead of the MMAs: poll the slot gently to leave issue slots to softmax
      ok = __all_sync(0xffffffffu, wait_l(&empty[slot], phase ^ 1u, abort, peer_abort, 128));
      if (!ok) return;
      int64_t* ids = ids_all + ((tile & 1) * kProducerWarps + pw) * 32;
      if (!isv) {  // resolve this tile's slot ids (used by K now and by V later)
        const int64_t raw = raw_q[0];
#pragma unroll
        for (int i = 0; i + 1 < kPrefetch; ++i) raw_q[i] = raw_q[i + 1];
        raw_q[kPrefetch - 1] = tile + kPrefetch < ntiles ? raw_of(tile + kPrefetch) : 0;
        ids[lane] = resolve_slot(raw, a.num_slots, a.slot_mode, a.err);
        __syncwarp();
      }
      const uint32_t sb = base + C::kOffRing + slot * C::kSlotBytes;
      if (!isv) {  // 16 key rows of D dims
        constexpr int CPR = D / 8, RPI = 32 / CPR;
        const int sub = lane / CPR, ch = lane - (lane / CPR) * CPR;
#pragma unroll
        for (int i = 0; i < 16; i += RPI) {
          const int kr = 16 * pw + i + sub;  // row in this CTA's K half
          const int64_t sl = ids[i + sub];
          cp_async16(sb + (ch >> 3) * C::kKBlk + kr * 128 + (((ch & 7) ^ (kr & 7)) << 4),
                     kbuf + sl * sstride + ch * 16);
        }
      } else {  // 32 key rows of this CTA's D/2 dims
        constexpr int CPR = D / 16, RPI = 32 / CPR;
        const int sub = lane / CPR, ch = lane - (lane / CPR) * CPR;
#pragma unroll
        for (int i = 0; i < 32; i += RPI) {
          const int idx = i + sub;
          const int vr = idx < 16 ? 64 * (int)rank + 16 * pw + idx : 64 * (1 - (int)rank) + 16 * pw + idx - 16;
          const int64_t sl = ids[idx];
          cp_async16(sb + (ch >> 3) * C::kVBlk + vr * 128 + (((ch & 7) ^ (vr & 7)) << 4),
                     vbuf + sl * sstride + ch * 16);
        }
      }
      cp_async_arrive_noinc(&full[slot]);
      if (++slot == C::kSlots) { slot = 0; phase ^= 1u; }
    };
    produce(0, false);
    if (ok && ntiles > 1) produce(1, false);
    for (int j = 0; ok && j < ntiles; ++j) {
      produce(j, true);
      if (ok && j + 2 < ntiles) produce(j + 2, false);
    }
    // Output gate, off the softmax's critical path: once the last S MMA has completed (q_dead), the
    // Q region is free; each producer warp copies 32 gate rows of this CTA into it (whole rows,
    // coalesced; the 16-byte chunks XOR-swizzled by the row) while the last tiles still run.  Every
    // producer thread reaches the closing barrier.
    const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
    const bool gated = a.gate_mode != TF_GATE_NONE && gate != nullptr && gate_vec(a);
    constexpr int kChunks = D / 8, kRowsPerInstr = 32 / kChunks;
    const int gsub = lane / kChunks, gch = lane - (lane / kChunks) * kChunks;
    bool okg = ok && wait_l(q_dead, 0, abort, peer_abort);
    okg = __all_sync(0xffffffffu, okg);
    if (okg && gated) {
#pragma unroll 1
      for (int i = 0; i < 32; i += kRowsPerInstr) {
        const int row = pw * 32 + i + gsub;
        const int ti = row / G, g = row - (row / G) * G;
        if (ti < n_tok)
          cp_async16(base + row * (D * 2) + ((gch ^ (row & (kChunks - 1))) << 4),
                     gate + (q0 + ti) * a.gate_stride_tok + (int64_t)(h * G + g) * a.gate_stride_head + gch * 8);
      }
    }
    cp_async_wait_all();
    named_barrier(6, (kSmWarps + kProducerWarps) * 32);  // gate rows staged for the softmax warps
  } else if (warp == kIssueWarp && rank == 1) {
    // ======================= relay: this CTA's halves landed -> rank 0 =======================
    if (lane == 0) {
      bool ok = wait_l(q_full, 0, abort, peer_abort);
      if (ok) {
        tc::fence_proxy_async_smem();
        remote_arrive(peer_addr(smem_u32(q_full), 0));
      }
      int slot = 0;
      uint32_t phase = 0;
      for (int it = 0; ok && it < 2 * ntiles; ++it) {
        ok = wait_l(&full[slot], phase, abort, peer_abort);
        if (!ok) break;
        tc::fence_proxy_async_smem();
        remote_arrive(peer_addr(smem_u32(&full[slot]), 0));
        if (++slot == C::kSlots) { slot = 0; phase ^= 1u; }
      }
      // rank 0's MMAs done with this CTA's TMEM and smem; waited for also after an abort (bounded)
      mbar_wait(fin, 0);
    }
    __syncwarp();
  } else if (warp == kFwdWarp) {
    // =========== rank 1: "this CTA's P_j is in TMEM" -> rank 0's p_full, one arrive per tile ===========
    if (rank == 1 && lane == 0) {
      const uint32_t pf0 = peer_addr(smem_u32(&p_full[0]), 0), pf1 = peer_addr(smem_u32(&p_full[1]), 0);
      for (int j = 0; j < ntiles; ++j) {
        if (!wait_l(&p_full[j & 1], (j >> 1) & 1, abort, peer_abort)) break;
        tc::fence_after_sync();
        tc::fence_before_sync();
        remote_arrive((j & 1) ? pf1 : pf0);
      }
    }
    __syncwarp();
  } else if (warp == kIssueWarp) {
    // ======================= MMA issue for the pair (rank 0, one thread) =======================
    if (lane == 0) {
      constexpr uint32_t kIdS = tc::idesc_bf16(2 * kRows, kPBN, false, false);
      constexpr uint32_t kIdO = tc::idesc_bf16(2 * kRows, D, false, true);
      bool ok = wait_c(q_full, 0, abort, peer_abort);
      tc::fence_proxy_async_smem();
      int slot = 0;
      uint32_t phase = 0;
      auto take = [&]() -> uint32_t {
        ok = ok && wait_c(&full[slot], phase, abort, peer_abort);
        tc::fence_proxy_async_smem();
        return base + C::kOffRing + slot * C::kSlotBytes;
      };
      auto release = [&]() {
        commit_both(&empty[slot]);
        if (++slot == C::kSlots) { slot = 0; phase ^= 1u; }
      };
      auto issue_s = [&](int t) {
        const uint32_t kb = take();
        if (!ok) return;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::sw128_desc(base + (kk >> 2) * C::kQBlock + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sw128_desc(kb + (kk >> 2) * C::kKBlk + (kk & 3) * 32, 16, 1024);
          mma2_ss(tmem + C::kColS + (t & 1) * kPBN, ad, bd, kIdS, kk > 0);
        }
        commit_both(&s_full[t & 1]);
        if (t == ntiles - 1) commit_both(q_dead);
        release();
      };
      auto issue_pv = [&](int t) {
        ok = ok && wait_c(&p_full[t & 1], (t >> 1) & 1, abort, peer_abort);
        tc::fence_after_sync();
        const uint32_t vb = take();
        if (!ok) return;
#pragma unroll
        for (int kk = 0; kk < kPBN / 16; ++kk) {
          // P_j: keys [64 hf, 64 hf + 64) packed in columns [64 hf, 64 hf + 32) of S buffer j & 1
          const uint64_t bd = tc::sw128_desc(vb + kk * 2048, C::kVBlk, 1024);
          mma2_ts(tmem + C::kColO, tmem + C::kColS + (t & 1) * kPBN + 64 * (kk >> 2) + (kk & 3) * 8, bd,
                  kIdO, t > 0 || kk > 0);
        }
        commit_both(o_done);
        release();
      };
      if (ok) issue_s(0);
      if (ok && ntiles > 1) issue_s(1);
      for (int j = 0; ok && j < ntiles; ++j) {
        issue_pv(j);
        if (ok && j + 2 < ntiles) issue_s(j + 2);
      }
      if (!ok) commit_both(q_dead);  // aborted before the last S: release the waiters anyway
      commit_both(fin);  // completes once every MMA issued above has completed
      // waited for also after an abort (bounded): no MMA may be in flight when TMEM is released
      drain_c(fin, 0);
    }
    __syncwarp();
  } else if (warp < kSmWarps) {
    // ============ softmax + epilogue: thread (half, r) = key columns [64 half, +64) of row r ============
    const float c2 = a.scale * kLog2e;
    const int r = tid & (kRows - 1);
    const int half = tid >> 7;
    const int ri = r / G;
    const bool row_valid = ri < n_tok;
    const int64_t klim = P + cta_start + ri + 1;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    constexpr int kOHalf = D / 2;  // O columns rescaled and stored by this thread
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;
    // No early exit from this loop: the two warps of a row group meet at a barrier every tile, so
    // a failed wait only turns the remaining iterations into barrier-only ones.
    for (int j = 0; j < ntiles; ++j) {
      const int bi = j & 1;
      if (ok) ok = __all_sync(0xffffffffu, wait_l(&s_full[bi], (j >> 1) & 1, abort, peer_abort));
      float s[2][32];
      float pm = -INFINITY;
      if (ok) {
        tc::fence_after_sync();
        const uint32_t sa = tmem + lane_base + C::kColS + bi * kPBN + 64 * half;
        tc::ld32(sa, s[0]);
        tc::ld32(sa + 32, s[1]);
        tc::wait_ld();
        // keys [0, vis) of this thread's 64 are visible to the row (0 for rows past the request end)
        const int64_t rem = row_valid ? klim - (int64_t)j * kPBN - 64 * half : 0;
        const int vis = rem <= 0 ? 0 : (rem >= 64 ? 64 : (int)rem);
        if (vis < 64) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int k = 0; k < 32; ++k)
              if (hh * 32 + k >= vis) s[hh][k] = -INFINITY;
        }
        pm = max_of_64(s);
      }
      // the row max over both halves (raw scores; c2 > 0)
      pmax[(bi * 2 + half) * kRows + r] = pm;
      named_barrier(1 + (warp & 3), 64);
      const float pm_other = pmax[(bi * 2 + (half ^ 1)) * kRows + r];
      if (!ok) continue;
      const float tmax = fmaxf(pm, pm_other) * c2;
      const bool need = tmax > m_used + kRescaleLog2 || (m_used == -INFINITY && tmax > -INFINITY);
      const float m_new = need ? tmax : m_used;
      const float alpha = need ? (m_used == -INFINITY ? 0.f : exp2f(m_used - m_new)) : 1.f;
      m_used = m_new;
      l_sum *= alpha;
      if (j > 0 && __any_sync(0xffffffffu, need)) {  // rescale this thread's half of its O row
        ok = __all_sync(0xffffffffu, wait_l(o_done, (j - 1) & 1, abort, peer_abort));
        if (!ok) continue;
        tc::fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < kOHalf / 32; ++cc) {
          const uint32_t ta = tmem + lane_base + C::kColO + half * kOHalf + cc * 32;
          float o[32];
          tc::ld32(ta, o);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] *= alpha;
          tc::st32(ta, o);
        }
      }
      const float nmu = m_used == -INFINITY ? 0.f : -m_used;
      float pk[32];
      l_sum += exp_pack(s[0], c2, nmu, *reinterpret_cast<float(*)[16]>(&pk[0])) +
               exp_pack(s[1], c2, nmu, *reinterpret_cast<float(*)[16]>(&pk[16]));
      // P over the first 32 of this thread's 64 S columns: only this thread read them
      tc::st32(tmem + lane_base + C::kColS + bi * kPBN + 64 * half, pk);
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[bi]);  // rank 1's warp 13 forwards it to rank 0
    }
    constexpr int kChunks = D / 8;                           // 16-byte chunks of a row
    constexpr int kRowsPerInstr = 32 / kChunks;              // 1 (D 256) or 2 (D 128)
    constexpr int kRowsPerWarp = kRows / kSmWarps;           // 16
    constexpr int kRowIters = kRowsPerWarp / kRowsPerInstr;
    const int sub = lane / kChunks, ch = lane - (lane / kChunks) * kChunks;
    const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    const bool gated = a.gate_mode != TF_GATE_NONE && gate != nullptr;
    const bool vec = gate_vec(a);
    const uint32_t gstage = base;  // gate rows, staged in the Q region by the producers
    if (ok) ok = __all_sync(0xffffffffu, wait_l(fin, 0, abort, peer_abort));
    // ---- epilogue.  Once fin completed, no MMA reads Q or the ring any more: the two halves' row
    // sums meet in the ring.  Every softmax thread reaches every barrier of its path.
    float* l_part = reinterpret_cast<float*>(sbase + C::kOffRing + kRows * D * 2);  // after the O stage
    if (ok) l_part[half * kRows + r] = l_sum;
    named_barrier(5, kSmWarps * 32);
    const float l_tot = ok ? l_part[r] + l_part[kRows + r] : 0.f;
    const uint32_t stage = base + C::kOffRing;
    if (vec) {
      // 16-byte gate and output pieces: each thread writes its own row's half straight from TMEM,
      // out = bf16(bf16(O / l) * bf16(act(gate))) (a bf16 x bf16 product is exact in fp32), with
      // the gate row read from the producers' staging (16-byte chunks XOR-swizzled by the row, so
      // the 32 rows of a warp read conflict-free)
      named_barrier(6, (kSmWarps + kProducerWarps) * 32);  // gate rows are staged
      if (ok) {
        tc::fence_after_sync();
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        const int g = r - ri * G;
        __nv_bfloat16* orow =
            row_valid ? out + (q0 + ri) * a.out_stride_tok + (int64_t)(h * G + g) * a.out_stride_head +
                            half * kOHalf
                      : nullptr;
#pragma unroll 1
        for (int cc = 0; cc < kOHalf / 32; ++cc) {
          float o[32];
          tc::ld32(tmem + lane_base + C::kColO + half * kOHalf + cc * 32, o);
          uint32_t gw[4][4];
          if (gated && row_valid) {
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
              const int chunk = (half * kOHalf + cc * 32) / 8 + c8;
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(gw[c8][0]), "=r"(gw[c8][1]), "=r"(gw[c8][2]), "=r"(gw[c8][3])
                           : "r"(gstage + r * (D * 2) + ((chunk ^ (r & (kChunks - 1))) << 4)));
            }
          }
          tc::wait_ld();
          if (row_valid) {
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
              uint4 ov;
              uint32_t* w = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
              for (int q2 = 0; q2 < 4; ++q2) {
                const float x0 = l_tot > 0.f ? o[c8 * 8 + 2 * q2] * inv : NAN;
                const float x1 = l_tot > 0.f ? o[c8 * 8 + 2 * q2 + 1] * inv : NAN;
                __nv_bfloat162 pv = __floats2bfloat162_rn(x0, x1);
                if (gated) {
                  const __nv_bfloat162 gv = *reinterpret_cast<const __nv_bfloat162*>(&gw[c8][q2]);
                  const __nv_bfloat162 av = __floats2bfloat162_rn(
                      act_fast(__low2float(gv), a.gate_mode), act_fast(__high2float(gv), a.gate_mode));
                  pv = __hmul2(pv, av);
                }
                w[q2] = *reinterpret_cast<uint32_t*>(&pv);
              }
              *reinterpret_cast<uint4*>(orow + cc * 32 + c8 * 8) = ov;
            }
          }
        }
      }
    } else {
      // unaligned gate or output rows: O (normalised, bf16) is staged row-major in the ring with
      // the 16-byte chunk index XOR-swizzled by the row, then written element by element
      if (ok) {
        tc::fence_after_sync();
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll 1
        for (int cc = 0; cc < kOHalf / 32; ++cc) {
          float o[32];
          tc::ld32(tmem + lane_base + C::kColO + half * kOHalf + cc * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint32_t w[4];
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
              const float x0 = l_tot > 0.f ? o[c8 * 8 + 2 * q2] * inv : NAN;
              const float x1 = l_tot > 0.f ? o[c8 * 8 + 2 * q2 + 1] * inv : NAN;
              __nv_bfloat162 pv = __floats2bfloat162_rn(x0, x1);
              w[q2] = *reinterpret_cast<uint32_t*>(&pv);
            }
            const int chunk = (half * kOHalf + cc * 32 + c8 * 8) / 8;
            const uint32_t dst = stage + r * (D * 2) + ((chunk ^ (r & (kChunks - 1))) << 4);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(w[0]), "r"(w[1]),
                         "r"(w[2]), "r"(w[3])
                         : "memory");
          }
        }
      }
      named_barrier(5, kSmWarps * 32);
      named_barrier(6, (kSmWarps + kProducerWarps) * 32);  // the producers' closing barrier
    }
    if (!vec && ok) {
#pragma unroll 1
      for (int i = 0; i < kRowIters; ++i) {
        const int row = warp * kRowsPerWarp + i * kRowsPerInstr + sub;
        const int ti = row / G, g = row - (row / G) * G;
        if (ti >= n_tok) continue;
        const int64_t t = q0 + ti;
        const int hq = h * G + g;
        const uint32_t src = stage + row * (D * 2) + ((ch ^ (row & (kChunks - 1))) << 4);
#pragma unroll 1
        for (int k = 0; k < 8; ++k) {
          unsigned short bits;
          asm volatile("ld.shared.u16 %0, [%1];" : "=h"(bits) : "r"(src + 2 * k));
          float v = __bfloat162float(__ushort_as_bfloat16(bits));
          if (gated)
            v = apply_gate<__nv_bfloat16>(
                v, to_f(gate[t * a.gate_stride_tok + (int64_t)hq * a.gate_stride_head + ch * 8 + k]),
                a.gate_mode);
          out[t * a.out_stride_tok + (int64_t)hq * a.out_stride_head + ch * 8 + k] = __float2bfloat16_rn(v);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  // rank 0's MMAs read this CTA's shared memory and TMEM, and remote arrivals target rank 0's
  // barriers: neither CTA releases TMEM or exits before both are done
  cluster_sync();
  if (tid == 0 && *abort) record_err(a.err, TF_KERR_TIMEOUT);
  tc::fence_after_sync();
  if (warp == kIssueWarp)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols)
                 : "memory");
}

template <int D>
static cudaError_t launch_pair(const tf_paged_attn_args& a, cudaStream_t s) {
  const int G = a.num_q_heads / a.num_kv_heads;
  const int TQ = kRows / G;
  const int pairs = (a.max_extend_len + 2 * TQ - 1) / (2 * TQ);
  cudaError_t e = cudaFuncSetAttribute(extend_pair_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)(2 * a.batch_size * pairs), (unsigned)a.num_kv_heads);
  extend_pair_kernel<D><<<grid, kPairThreads, Cfg<D>::kSmem, s>>>(a, pairs);
  return cudaGetLastError();
}

}  // namespace pair
}  // namespace ext

bool paged_extend_tc_supported(const tf_paged_attn_args& a) {
  if (a.dtype != TF_DTYPE_BF16) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  const int G = a.num_q_heads / a.num_kv_heads;
  if (G < 1 || G > 16 || ext::kRows % G != 0) return false;
  if (a.max_extend_len <= 0) return false;
  if (!(a.scale > 0.f)) return false;  // the softmax takes its max on unscaled scores
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.q) || !al(a.k_buffer) || !al(a.v_buffer)) return false;
  if (a.q_stride_tok % 8 || a.q_stride_head % 8 || a.kv_stride_slot % 8 || a.kv_stride_head % 8)
    return false;
  return true;
}

cudaError_t launch_paged_extend_tc(const tf_paged_attn_args& a, cudaStream_t s) {
  if (a.batch_size == 0 || a.num_tokens == 0) return cudaSuccess;
  switch (a.head_dim) {
    case 64: return ext::launch_d<64>(a, s);
    case 128: return ext::pair::launch_pair<128>(a, s);
    default: return ext::pair::launch_pair<256>(a, s);
  }
}

}  // namespace tf
