// mmltk_msda_bwd_noalloc -- multi-scale deformable attention backward that
// allocates no memory.
//
// This entry point has no counterpart in the reference implementation.  It
// exists for callers that must not allocate GPU memory while they run: code
// that executes while a custom allocator or memory pool owns all device
// memory, inference/training runtimes that pre-plan every byte up front,
// and C/C++ hosts without PyTorch's caching allocator that cannot call
// cudaMalloc in their hot path (cudaMalloc synchronises the device and can
// fail late, after the caller has committed to the work).
//
// The caller passes every input and output buffer.  The fp32 accumulators
// the backward pass needs live in a fixed array inside this library
// (MMLTK_NOALLOC_MAX_VALUE_ELEMS + MMLTK_NOALLOC_MAX_REF_ELEMS floats, 36 MiB), which every
// GPU that loads the library keeps until the process exits.
//
// Set-up: the first call on a device looks up the array's device address
// (cudaGetSymbolAddress) with that device current; make that first call
// before capturing any stream into a CUDA graph.
//
// Sharing: every call uses the same array, and it keeps the previous call's
// contents (the accumulators are cleared at the start of each call).  Calls
// whose GPU work overlaps -- two streams, two host threads, or two devices
// sharing a context incorrectly -- race on the array; serialise them.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest problem the fixed scratch array holds.
#define MMLTK_NOALLOC_MAX_VALUE_ELEMS (8u * 1024u * 1024u)  // B*S*H*D   (value / grad_value elements)
#define MMLTK_NOALLOC_MAX_REF_ELEMS (1u * 1024u * 1024u)    // B*Lq*L*4  (reference-box elements)

// Return codes: 0 success; a positive value is a cudaError_t from the runtime;
// negative values are argument errors:
#define MMLTK_NOALLOC_ERR_TOO_LARGE (-1)   // problem exceeds the fixed scratch size
#define MMLTK_NOALLOC_ERR_BAD_ARG (-2)     // unsupported dtype / head dim / level or point count

// dtype: 0 = fp32, 1 = bf16 (all tensors share it).  Layouts (contiguous):
//   grad_out [B,Lq,H*D], value [B,S,H,D], shapes int32 [L,2] (h,w) and
//   starts int32 [L] on the device, ref [B,Lq,L,4] (cx,cy,w,h), offsets
//   [B,Lq,H,L,P,2] (raw sampling-offset outputs), logits [B,Lq,H,L*P] (raw
//   attention-weight outputs); outputs have the shapes of value, ref,
//   offsets and logits.  stream is a cudaStream_t (0 = legacy default stream).
int mmltk_msda_bwd_noalloc(int dtype, const void* grad_out, const void* value, const int* shapes, const int* starts,
                           const void* ref, const void* offsets, const void* logits, void* grad_value,
                           void* grad_ref, void* grad_offsets, void* grad_logits, int B, int S, int Lq, int H, int L,
                           int P, int D, void* stream);

#ifdef __cplusplus
}
#endif
