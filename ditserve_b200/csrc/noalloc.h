// Allocation-free C entry point of ditserve_b200 (exported from the _C extension library).
//
// DECLARATION: an addition of this project with no counterpart in the reference
// project.  It serves callers that may not allocate device memory (an embedding
// application that owns every byte of GPU memory in its own pool, a plugin inside
// another framework that accounts for all device memory, a serving loop that must
// not enter the driver allocator after start-up).  It runs the fused q/k RMS norm
// + RoPE + tcgen05 attention with its staging buffer in a fixed 16 MiB file-scope
// device array instead of cudaMalloc'd memory; see noalloc.cu for the full contract
// (size limit, 16-byte pointer alignment, supported widths, stream on the current
// device, shared array, first-call set-up, no overlapping calls).
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

enum {
  DS_NOALLOC_OK = 0,
  DS_NOALLOC_TOO_LARGE = 1,     // batch*seq*3*heads*head_dim*2 bytes exceed the 16 MiB array
  DS_NOALLOC_BAD_ARGUMENT = 2,  // null or misaligned pointer (16 bytes required), unsupported shape
                                // (head_dim 64/128; heads*head_dim in {512,1024,1536,2048,3072}),
                                // bad stride, or a stream of another device
  DS_NOALLOC_CUDA_ERROR = 3,    // the current device or the device array's address could not be obtained
  DS_NOALLOC_LAUNCH_ERROR = 4,  // a kernel launch of this call failed
  DS_NOALLOC_INTERNAL_ERROR = 5,  // host-side launch set-up failed (for example a tensor-map encode)
};

int ds_fused_qkv_attention_noalloc(const void* qkv, long long qkv_stride, int batch, int seq, int heads,
                                   int head_dim, const void* wq, const void* wk, float eps, const float* rope_cos,
                                   const float* rope_sin, void* out, long long out_stride, int* status,
                                   void* stream);

#ifdef __cplusplus
}
#endif
