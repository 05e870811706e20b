// Public C entry points of the paged attention kernels.
//
// Every function returns 0 on success, a CUDA error code, or a negative code of
// this library (shape or size rejected before anything is launched).  Parameter
// blocks are the plain structs of params.h; all pointers are device pointers.
#pragma once
#include <stddef.h>

#include "params.h"

extern "C" {

// Split-KV paged attention over the INT2 (kv_mode 0) or BF16 (kv_mode 1) cache:
// writes one partial (64 rows x D, fp32) and its log-sum-exps per (work item, KV head)
// into attn->part_o / attn->part_lse.
int oscar_paged_attention(const oscar::AttnParams* attn, cudaStream_t stream);

// Merges the partials of each query row, rotates back by R_v^T, applies the gate and
// writes bf16 and / or int8 + per-row scale outputs.
int oscar_attn_merge(const oscar::MergeParams* merge, cudaStream_t stream);

// Allocation-free attention.  This entry point has no counterpart in the reference.
//
// It is for callers that cannot allocate device memory at the time they run attention:
// code inside a custom allocator or memory-pool callback (allocating there re-enters
// the allocator), runtimes that forbid cudaMalloc on their serving path (it can
// synchronise the device and stall other streams), and embedders that must keep a
// memory footprint fixed at start-up.  It computes exactly what oscar_paged_attention
// followed by oscar_attn_merge computes, with the same inputs and outputs, but the
// split-KV partials go to a fixed device array inside this library instead of a
// caller workspace (the part_o / part_lse fields of both blocks are ignored).
//
//  * At most OSCAR_NOALLOC_MAX_ITEMS (work item x KV head) partials per call: 16 MiB of
//    fp32 partials plus 64 KiB of log-sum-exps.  Larger calls return -310 and launch
//    nothing.
//  * Every GPU that loads this library holds that array until the process exits.
//  * All calls on a device share the array and leave their contents in it.  Each call
//    writes every partial before it reads it, so nothing has to start at zero, but
//    calls whose kernels overlap on the GPU (streams with no ordering between them)
//    race on the array: the caller must serialise them.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call before
//    any stream capture.
//  * It calls no cudaMalloc, cudaFree or other allocating routine.
#define OSCAR_NOALLOC_MAX_ITEMS 256
int oscar_paged_attention_noalloc(const oscar::AttnParams* attn, const oscar::MergeParams* merge,
                                  cudaStream_t stream);

// The layout of the parameter blocks as compiled into this library, for callers that
// mirror the structs in another language (ctypes, cffi): writes up to `cap` values
// {sizeof(AttnParams), offsetof of each AttnParams field in declaration order,
//  sizeof(MergeParams), offsetof of each MergeParams field in declaration order}
// and returns how many values the full list has.
int oscar_params_layout(long long* out, int cap);

}  // extern "C"
