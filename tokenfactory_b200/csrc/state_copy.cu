// GDN state-slot copies (ReqToStatePool.capture_snapshot / restore_snapshot / reset_working_state /
// free_snapshot, req_to_state_pool.py:120-194) for all linear layers and both pools in one launch.
//
// Work is cut into units of one (op, pool, layer, 32 KB tile); every unit is a contiguous byte
// range of one slot of one layer (the reference's [L, slots, ...] layouts keep a slot's rows of a
// layer contiguous).  A persistent grid of a few CTAs per SM walks the units; each thread issues
// its 8 x 16-byte loads before its stores so that a CTA keeps 32 KB in flight.  HBM-bound: the
// algorithmic bytes are read + write of every copied byte (write only for zeroing).
#include "common.cuh"
#include "launch.h"

namespace tf {
namespace state_copy {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 8;
constexpr int64_t kTile = (int64_t)kThreads * kVecPerThread * 16;  // 32 KB

struct Pool {
  char* base;
  int64_t layer_bytes, slot_bytes, bytes;  // strides and the contiguous extent, in bytes
  int64_t tiles;                           // tiles per (slot, layer)
};

__device__ __forceinline__ bool slot_ok(int64_t s, int64_t n) { return s >= 0 && s < n; }

template <bool VEC>
__device__ __forceinline__ void copy_tile(const Pool& p, int64_t layer, int64_t src, int64_t dst,
                                          int64_t tile) {
  const int64_t off = tile * kTile;
  const int64_t n = p.bytes - off < kTile ? p.bytes - off : kTile;
  char* d = p.base + layer * p.layer_bytes + dst * p.slot_bytes + off;
  const char* s = src >= 0 ? p.base + layer * p.layer_bytes + src * p.slot_bytes + off : nullptr;
  if (VEC) {
    const int nv = (int)(n >> 4);
    uint4 v[kVecPerThread];
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int i = threadIdx.x + k * kThreads;
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (s && i < nv) v[k] = __ldcs(reinterpret_cast<const uint4*>(s) + i);
    }
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int i = threadIdx.x + k * kThreads;
      if (i < nv) __stcs(reinterpret_cast<uint4*>(d) + i, v[k]);
    }
  } else {
    for (int64_t i = threadIdx.x; i < n; i += kThreads) d[i] = s ? s[i] : (char)0;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) slots_copy_kernel(tf_state_copy_args a, Pool conv,
                                                              Pool ssm, int64_t units_per_op) {
  const int64_t L = a.num_layers;
  const int64_t conv_units = conv.base ? L * conv.tiles : 0;
  const int64_t total = units_per_op * a.num_ops;
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    const int64_t op = u / units_per_op;
    int64_t r = u - op * units_per_op;
    const int64_t src = a.src_slots[op], dst = a.dst_slots[op];
    if (!slot_ok(dst, a.num_slots) || (src != -1 && !slot_ok(src, a.num_slots))) {
      if (r == 0 && threadIdx.x == 0) record_err(a.err, TF_KERR_SLOT_RANGE);
      continue;
    }
    if (src == dst) continue;
    if (r < conv_units) {
      copy_tile<VEC>(conv, r / conv.tiles, src, dst, r % conv.tiles);
    } else {
      r -= conv_units;
      copy_tile<VEC>(ssm, r / ssm.tiles, src, dst, r % ssm.tiles);
    }
  }
}

inline int elem_bytes(int32_t dt) { return dt == TF_DTYPE_F32 ? 4 : 2; }

inline Pool make_pool(void* base, int64_t stride_layer, int64_t stride_slot, int64_t elems,
                      int32_t dt) {
  Pool p{};
  if (!base || elems <= 0) return p;
  const int eb = elem_bytes(dt);
  p.base = static_cast<char*>(base);
  p.layer_bytes = stride_layer * eb;
  p.slot_bytes = stride_slot * eb;
  p.bytes = elems * eb;
  p.tiles = (p.bytes + kTile - 1) / kTile;
  return p;
}

inline bool aligned16(const Pool& p) {
  if (!p.base) return true;
  return ((reinterpret_cast<uintptr_t>(p.base) | (uintptr_t)p.layer_bytes | (uintptr_t)p.slot_bytes |
           (uintptr_t)p.bytes) & 15) == 0;
}

}  // namespace state_copy

cudaError_t launch_state_slots_copy(const tf_state_copy_args& a, cudaStream_t s) {
  using namespace state_copy;
  const Pool conv = make_pool(a.conv_state, a.conv_stride_layer, a.conv_stride_slot,
                              a.conv_slot_elems, a.conv_dtype);
  const Pool ssm = make_pool(a.ssm_state, a.ssm_stride_layer, a.ssm_stride_slot,
                             a.ssm_slot_elems, a.ssm_dtype);
  const int64_t units_per_op = (int64_t)a.num_layers * (conv.tiles + ssm.tiles);
  const int64_t total = units_per_op * a.num_ops;
  if (total == 0) return cudaSuccess;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  const int grid = (int)(total < cap ? total : cap);
  if (aligned16(conv) && aligned16(ssm))
    slots_copy_kernel<true><<<grid, kThreads, 0, s>>>(a, conv, ssm, units_per_op);
  else
    slots_copy_kernel<false><<<grid, kThreads, 0, s>>>(a, conv, ssm, units_per_op);
  return cudaGetLastError();
}

}  // namespace tf
