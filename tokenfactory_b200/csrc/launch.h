// Internal launchers behind the C ABI (capi.cu validates arguments, then calls these).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "tfattn.h"

namespace tf {

// kv_store.cu
cudaError_t launch_kv_store(const tf_kv_store_args& a, cudaStream_t s);
// prologue.cu: fused q/k RMSNorm + partial RoPE + KV store
bool attn_prologue_supported(const tf_attn_prologue_args& a);
cudaError_t launch_attn_prologue(const tf_attn_prologue_args& a, cudaStream_t s);

// paged_attn_simt.cu: any dtype / head_dim <= 256, decode and extend
cudaError_t launch_paged_attn_simt(const tf_paged_attn_args& a, cudaStream_t s);

// paged_extend_tc.cu: bf16 extend on tcgen05 / TMEM
bool paged_extend_tc_supported(const tf_paged_attn_args& a);
cudaError_t launch_paged_extend_tc(const tf_paged_attn_args& a, cudaStream_t s);

// paged_decode_mma.cu: bf16 / fp16 decode on tensor cores, balanced split-KV.  Its combine kernel
// keeps the schedule (batch_size + 1 int32) in shared memory, so batches above kDecodeMmaMaxBatch
// take the CUDA-core kernel instead (checked before any launch).
constexpr int kDecodeMmaMaxBatch = 32768;
bool paged_decode_mma_supported(const tf_paged_attn_args& a);
size_t paged_decode_mma_workspace(const tf_paged_attn_args& a, int num_sms);
cudaError_t launch_paged_decode_mma(const tf_paged_attn_args& a, void* ws, size_t ws_bytes,
                                    int num_sms, cudaStream_t s);
// same kernels with the scratch in a fixed device array of kNoAllocScratchBytes (no allocation);
// cudaErrorStreamCaptureUnsupported when the stream is capturing and the array's address on the
// current device has not been resolved by an earlier call outside capture
constexpr size_t kNoAllocScratchBytes = 4u << 20;
cudaError_t launch_paged_decode_mma_noalloc(const tf_paged_attn_args& a, int num_sms,
                                            cudaStream_t s);

// gdn.cu
bool gdn_dims_supported(int dk, int dv);
cudaError_t launch_gdn_decode(const tf_gdn_args& a, cudaStream_t s);
size_t gdn_extend_workspace(const tf_gdn_args& a);
cudaError_t launch_gdn_extend(const tf_gdn_args& a, void* ws, size_t ws_bytes, cudaStream_t s);

// rmsnorm.cu
cudaError_t launch_gated_rmsnorm(const tf_gated_rmsnorm_args& a, cudaStream_t s);

// state_copy.cu: GDN state-slot snapshot copies / resets for all layers in one launch
cudaError_t launch_state_slots_copy(const tf_state_copy_args& a, cudaStream_t s);

// runtime.cu: per-step req_to_token sync and batched sampling
cudaError_t launch_req_to_token_sync(const tf_r2t_sync_args& a, cudaStream_t s);
cudaError_t launch_sample_tokens(const tf_sample_args& a, cudaStream_t s);

// fp8_gemm.cu: block-FP8 linear (activation quantization + tcgen05 kind::f8f6f4 GEMM)
cudaError_t launch_fp8_quantize(const tf_fp8_quant_args& a, cudaStream_t s);
cudaError_t launch_fp8_block_gemm(const tf_fp8_gemm_args& a, cudaStream_t s);

// capi.cu
int device_sm_count();

}  // namespace tf
