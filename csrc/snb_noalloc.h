// C interface of the allocation-free decode-attention entry point (csrc/kernels/attention_noalloc.cu).
//
// This interface has no counterpart in the reference; it is an addition of this library.
//
// It is for callers that cannot allocate device memory at the moment they run attention: code inside a
// memory-allocator callback or an out-of-memory handler (an allocation there would re-enter the allocator),
// runtimes whose device memory is reserved up front and handed out only as fixed buffers, and plain C/C++ or
// FFI hosts with no caching allocator to borrow temporary buffers from. The split-K scratch lives in a
// fixed-size device array inside the loaded library (4 MiB per GPU, held until the process exits), so a
// call takes only the caller's inputs and outputs.
//
// Limits and rules (details beside the definitions):
//  * scratch need = batch * num_q_heads * num_splits * (head_dim + 1) fp32 values, at most
//    snb_decode_attention_noalloc_scratch_capacity(); larger requests return SNB_NOALLOC_ERR_TOO_LARGE;
//  * the first call on a device (and the first after that device's context changed) looks up the array's
//    device address; make it outside any CUDA stream capture;
//  * every call shares the one array: calls that may overlap on the GPU race and must be serialised by the
//    caller (one stream, or explicit ordering);
//  * nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SNB_NOALLOC_OK = 0,
  SNB_NOALLOC_ERR_ARGS = -1,       // bad argument (null pointer, head_dim not 64/128, heads not divisible, ...)
  SNB_NOALLOC_ERR_TOO_LARGE = -2,  // scratch request above the fixed capacity; nothing launched
  SNB_NOALLOC_ERR_SYMBOL = -3,     // the device address of the scratch array could not be looked up
  SNB_NOALLOC_ERR_LAUNCH = -4,     // a kernel launch of this call failed
  SNB_NOALLOC_ERR_PRIOR = -5,      // an earlier CUDA error was already pending on this thread; nothing launched
};

// Largest scratch request accepted, in fp32 values.
long long snb_decode_attention_noalloc_scratch_capacity(void);

// Paged decode attention (one new query per request) that allocates nothing. Device pointers; `stream` may
// be 0. q: [batch, num_q_heads * head_dim] bf16 rows of stride q_stride; k_cache/v_cache:
// [pages, num_kv_heads, page_size, head_dim], bf16 or fp8 e4m3 (kv_fp8 = 1) with k_scale/v_scale;
// block_table: [batch, block_table_stride] int32 page ids; seq_lens: [batch] int32 context lengths (0 allowed);
// window > 0 keeps only the last `window` positions; sinks: [num_q_heads] fp32 or null; out: [batch,
// num_q_heads * head_dim] bf16 rows of stride out_stride. Returns SNB_NOALLOC_OK or a negative code above.
int snb_decode_attention_noalloc(void* out, int out_stride, const void* q, int q_stride, const void* k_cache,
                                 const void* v_cache, int kv_fp8, const int32_t* block_table,
                                 int block_table_stride, const int32_t* seq_lens, int batch, int num_q_heads,
                                 int num_kv_heads, int head_dim, int page_size, int window, float sm_scale,
                                 float k_scale, float v_scale, const float* sinks, int num_splits,
                                 cudaStream_t stream);

#ifdef __cplusplus
}
#endif
