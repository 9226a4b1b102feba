// a3 + a4: paged GQA extend / prefill attention over a radix-cached prefix on the 5th-generation
// tensor cores (qwen3_8/full_attention.py:179-213 and :244-283, output gate :157-158).
//
// One CTA (one warpgroup, 128 threads) owns 128 query rows: 128/G consecutive query tokens of one
// request times the G query heads that share kv head h (GQA packed into M).  Q stays resident in
// shared memory (SWIZZLE_128B, K-major).  Keys are visited in tiles of 64 token rows gathered
// through req_to_token by cp.async into a double-buffered SWIZZLE_128B ring (K and V with the same
// physical layout: K is read K-major, V MN-major).  Per tile:
//   S = Q.K^T      tcgen05.mma M128 N64 K16 x D/16 -> TMEM (64 fp32 columns)
//   softmax        thread r owns row r: tcgen05.ld of its 64 scores, causal mask, online max/sum
//                  with a lazy rescale (O in TMEM is rescaled only when a row's max grows by more
//                  than 2^8), P in bf16 written to shared memory (SWIZZLE_128B, K-major)
//   O += P.V       tcgen05.mma M128 N=D K16 x 4 -> TMEM (D fp32 columns)
// Completion of each MMA group is tracked with tcgen05.commit on an mbarrier; every wait is
// bounded.  The epilogue reads O from TMEM, divides by the row sum, applies the output gate and
// stores bf16.  Rows past the end of the request and keys outside a row's causal window are
// masked; query i of request b sees keys j <= seq_len - extend_len + i.
#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace tf {
namespace ext {

constexpr int kRows = 128;
constexpr int kBN = 64;
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;

template <int D>
struct Cfg {
  static constexpr int kKB = D / 64;             // 64-element blocks of a row
  static constexpr int kQBlock = kRows * 128;    // one 64-dim block of Q
  static constexpr int kKVBlock = kBN * 128;     // one 64-dim block of a K or V tile
  static constexpr int kQBytes = kKB * kQBlock;
  static constexpr int kKBytes = kKB * kKVBlock;
  static constexpr int kStage = 2 * kKBytes;     // K tile then V tile
  static constexpr int kPBytes = kRows * 128;    // P: 128 rows x 64 keys bf16
  static constexpr int kOffKV = kQBytes;
  static constexpr int kOffP = kOffKV + 2 * kStage;
  static constexpr int kOffMisc = kOffP + kPBytes;   // barriers, TMEM holder, slot ids
  static constexpr int kMiscBytes = 64 + 2 * kBN * 8;
  static constexpr int kSmem = kOffMisc + kMiscBytes + 1024;  // + slack to align the base
  static constexpr int kColO = kBN;
  static constexpr int kTmemCols = (kBN + D) <= 256 ? 256 : 512;
  static_assert(D % 64 == 0, "head_dim multiple of 64");
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    extend_kernel(tf_paged_attn_args a, int tiles_per_req) {
  using C = Cfg<D>;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023) & ~1023u;
  unsigned char* sbase = smem_raw + (base - raw_base);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sbase + C::kOffMisc);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar_s + 2);
  int64_t* slot_s = reinterpret_cast<int64_t*>(sbase + C::kOffMisc + 64);  // [2][kBN]

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
    if (threadIdx.x == 0) record_err(a.err, TF_KERR_SLOT_RANGE);
    return;
  }
  const int64_t P = L - E;
  const int n_tok = (int)(E - tile_start < TQ ? E - tile_start : TQ);
  const int64_t kv_end = P + tile_start + n_tok;  // keys [0, kv_end) are visible to some row
  const int ntiles = (int)((kv_end + kBN - 1) / kBN);

  // token offset of request b (exclusive prefix of extend_lens), by warp 0
  __shared__ int64_t s_q0;
  if (warp == 0) {
    int64_t acc = 0;
    for (int i = lane; i < b; i += 32) acc += a.extend_lens ? a.extend_lens[i] : 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s_q0 = acc;
  }
  int64_t row = a.req_pool_indices[b];
  if (row < 0 || row >= a.r2t_rows) {
    if (tid == 0) record_err(a.err, TF_KERR_REQ_RANGE);
    row = 0;
  }
  const int64_t* r2t = a.req_to_token + row * a.r2t_stride;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_holder, C::kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const int64_t q0 = s_q0 + tile_start;

  // ---- Q tile -> shared memory (rows past the request end are zero)
  {
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q);
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    for (int e = tid; e < kRows * CPR; e += kThreads) {
      const int r = e / CPR, ch = e - (e / CPR) * CPR;
      const int i = r / G, g = r - (r / G) * G;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (i < n_tok)
        v = *reinterpret_cast<const uint4*>(q + (q0 + i) * a.q_stride_tok +
                                            (int64_t)(h * G + g) * a.q_stride_head + ch * 8);
      const uint32_t dst = base + (ch >> 3) * C::kQBlock + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(v.x), "r"(v.y),
                   "r"(v.z), "r"(v.w)
                   : "memory");
    }
  }

  const char* kbuf = (const char*)a.k_buffer + (int64_t)h * a.kv_stride_head * 2;
  const char* vbuf = (const char*)a.v_buffer + (int64_t)h * a.kv_stride_head * 2;
  const int64_t sstride = a.kv_stride_slot * 2;
  auto raw_slot = [&](int tile) -> int64_t {  // threads < kBN: key tile*64 + tid
    int64_t key = (int64_t)tile * kBN + tid;
    if (key >= kv_end) key = (int64_t)tile * kBN;  // past the window: repeat the tile's first key
    return r2t[key];
  };
  auto issue_tile = [&](int tile, int buf, int64_t raw) {
    if (tid < kBN) slot_s[buf * kBN + tid] = resolve_slot(raw, a.num_slots, a.slot_mode, a.err);
    __syncthreads();
    constexpr int CPR = D / 8;
    const uint32_t st = base + C::kOffKV + buf * C::kStage;
    for (int e = tid; e < 2 * kBN * CPR; e += kThreads) {
      const int isv = e / (kBN * CPR);
      const int rem = e - isv * (kBN * CPR);
      const int key = rem / CPR, ch = rem - (rem / CPR) * CPR;
      const char* src = (isv ? vbuf : kbuf) + slot_s[buf * kBN + key] * sstride + ch * 16;
      const uint32_t dst = st + isv * C::kKBytes + (ch >> 3) * C::kKVBlock + key * 128 +
                           (((ch & 7) ^ (key & 7)) << 4);
      cp_async16(dst, src);
    }
    (void)tile;
  };

  const float c2 = a.scale * kLog2e;
  const int r = tid;                 // this thread's row == TMEM lane
  const int ri = r / G, rg = r - (r / G) * G;
  const bool row_valid = ri < n_tok;
  const int64_t klim = P + tile_start + ri + 1;  // keys [0, klim) visible to this row
  float m_used = -INFINITY, l_sum = 0.f;
  constexpr uint32_t kIdS = tc::idesc_bf16(kRows, kBN, false, false);
  constexpr uint32_t kIdO = tc::idesc_bf16(kRows, D, false, true);
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  int64_t next_raw = tid < kBN ? raw_slot(0) : 0;
  issue_tile(0, 0, next_raw);
  asm volatile("cp.async.commit_group;" ::: "memory");
  next_raw = (tid < kBN && ntiles > 1) ? raw_slot(1) : 0;

  // Only thread 0 waits on the MMA barriers (bounded); it publishes the outcome in s_ok before a
  // CTA barrier, so every thread takes the same exit, and the others order their TMEM accesses
  // after that barrier with tcgen05.fence::after_thread_sync.
  __shared__ int s_ok;
  if (tid == 0) s_ok = 1;
  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (tid == 0 && j >= 1 && !mbar_wait(bar_o, (j - 1) & 1)) s_ok = 0;  // PV_{j-1} done
    __syncthreads();
    if (!s_ok) break;
    tc::fence_after_sync();
    if (j + 1 < ntiles) {
      issue_tile(j + 1, buf ^ 1, next_raw);
      next_raw = (tid < kBN && j + 2 < ntiles) ? raw_slot(j + 2) : 0;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    tc::fence_proxy_async_smem();
    __syncthreads();

    // ---- S = Q . K_j^T
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t kb = base + C::kOffKV + buf * C::kStage;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t ad = tc::sw128_desc(base + (kk >> 2) * C::kQBlock + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = tc::sw128_desc(kb + (kk >> 2) * C::kKVBlock + (kk & 3) * 32, 16, 1024);
        tc::mma_bf16(tmem, ad, bd, kIdS, kk > 0);
      }
      tc::commit(bar_s);
      if (!mbar_wait(bar_s, j & 1)) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) break;
    tc::fence_after_sync();

    // ---- online softmax of row r over this tile's 64 keys
    float s[2][32];
    tc::ld32(tmem + lane_base + 0, s[0]);
    tc::ld32(tmem + lane_base + 32, s[1]);
    tc::wait_ld();
    const int64_t key0 = (int64_t)j * kBN;
    float tmax = -INFINITY;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const bool v = row_valid && key0 + hh * 32 + k < klim;
        s[hh][k] = v ? s[hh][k] * c2 : -INFINITY;
        tmax = fmaxf(tmax, s[hh][k]);
      }
    const bool need = tmax > m_used + kRescaleLog2 || (m_used == -INFINITY && tmax > -INFINITY);
    const float m_new = need ? tmax : m_used;
    const float alpha = need ? (m_used == -INFINITY ? 0.f : exp2f(m_used - m_new)) : 1.f;
    m_used = m_new;
    l_sum *= alpha;
    if (j > 0 && __any_sync(0xffffffffu, need)) {  // rescale O rows of this warp (TMEM)
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        tc::ld32(tmem + lane_base + C::kColO + cc * 32, o);
        tc::wait_ld();
#pragma unroll
        for (int k = 0; k < 32; ++k) o[k] *= alpha;
        tc::st32(tmem + lane_base + C::kColO + cc * 32, o);
      }
      tc::wait_st();
    }
    // P (bf16) -> shared memory, row r, SWIZZLE_128B
    const uint32_t prow = base + C::kOffP + r * 128;
#pragma unroll
    for (int cch = 0; cch < 8; ++cch) {
      uint32_t w[4];
#pragma unroll
      for (int q2 = 0; q2 < 4; ++q2) {
        const int k = cch * 8 + q2 * 2;
        const float x0 = s[k >> 5][k & 31], x1 = s[(k + 1) >> 5][(k + 1) & 31];
        const float p0 = x0 == -INFINITY ? 0.f : exp2f(x0 - m_used);
        const float p1 = x1 == -INFINITY ? 0.f : exp2f(x1 - m_used);
        l_sum += p0 + p1;
        __nv_bfloat162 pv = __floats2bfloat162_rn(p0, p1);
        w[q2] = *reinterpret_cast<uint32_t*>(&pv);
      }
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(prow + ((cch ^ (r & 7)) << 4)),
                   "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    // ---- O (+)= P . V_j
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t vb = base + C::kOffKV + buf * C::kStage + C::kKBytes;
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk) {
        const uint64_t ad = tc::sw128_desc(base + C::kOffP + kk * 32, 16, 1024);
        const uint64_t bd = tc::sw128_desc(vb + kk * 2048, C::kKVBlock, 1024);
        tc::mma_bf16(tmem + C::kColO, ad, bd, kIdO, j > 0 || kk > 0);
      }
      tc::commit(bar_o);
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  // the last PV must be complete before TMEM is read or released (bounded wait, thread 0)
  if (tid == 0) {
    if (!mbar_wait(bar_o, (ntiles - 1) & 1)) s_ok = 0;
    if (!s_ok) record_err(a.err, TF_KERR_TIMEOUT);
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  tc::fence_after_sync();

  // ---- epilogue: O / l, output gate, bf16
  if (ok) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
    const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
    const int64_t t = q0 + ri;
    const int hq = h * G + rg;
#pragma unroll 1
    for (int cc = 0; cc < D / 32; ++cc) {
      float o[32];
      tc::ld32(tmem + lane_base + C::kColO + cc * 32, o);
      tc::wait_ld();
      if (row_valid) {
        __nv_bfloat16* op = out + t * a.out_stride_tok + (int64_t)hq * a.out_stride_head + cc * 32;
        const __nv_bfloat16* gp =
            gate ? gate + t * a.gate_stride_tok + (int64_t)hq * a.gate_stride_head + cc * 32 : nullptr;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          float v = round_to<__nv_bfloat16>(l_sum > 0.f ? o[k] * inv : NAN);
          if (a.gate_mode != TF_GATE_NONE && gp != nullptr)
            v = apply_gate<__nv_bfloat16>(v, to_f(gp[k]), a.gate_mode);
          op[k] = __float2bfloat16_rn(v);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, C::kTmemCols);
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

}  // namespace ext

bool paged_extend_tc_supported(const tf_paged_attn_args& a) {
  if (a.dtype != TF_DTYPE_BF16) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  const int G = a.num_q_heads / a.num_kv_heads;
  if (G < 1 || G > 16 || ext::kRows % G != 0) return false;
  if (a.max_extend_len <= 0) return false;
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
    case 128: return ext::launch_d<128>(a, s);
    default: return ext::launch_d<256>(a, s);
  }
}

}  // namespace tf
