// Shared device helpers for the oscar_b200 kernels (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "oscar_b200 kernels are written for sm_100a (B200) only"
#endif

#define OSCAR_DEVICE __device__ __forceinline__

namespace oscar {

// Error codes written to the per-launch status word when a bounded wait expires
// or a bounds check fails.  The host reads the word after the step; a non-zero
// value fails the request/engine with a clear message instead of hanging a GPU.
enum StatusCode : int {
  kOk = 0,
  kTimeoutTmaFull = 1,
  kTimeoutSlotEmpty = 2,
  kTimeoutAccFull = 3,
  kTimeoutAccEmpty = 4,
  kTimeoutPeerFlag = 5,
  kBadBlockIndex = 16,
  kBadSlot = 17,
  kBadShape = 18,
};

OSCAR_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
OSCAR_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
OSCAR_DEVICE int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions for blockDim.x <= 1024 (result valid in every thread).
template <int NWARPS>
OSCAR_DEVICE float block_sum(float v, float* smem /* NWARPS floats */) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) smem[w] = v;
  __syncthreads();
  float t = (l < NWARPS) ? smem[l] : 0.f;
  return warp_sum(t);
}
template <int NWARPS>
OSCAR_DEVICE float block_max(float v, float* smem) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) smem[w] = v;
  __syncthreads();
  float t = (l < NWARPS) ? smem[l] : -INFINITY;
  return warp_max(t);
}

OSCAR_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Lets the next kernel of the stream start its CTAs now if it was launched as a
// programmatic dependent (the W8A8 GEMM is): it waits for this kernel's completion
// before it reads what this kernel writes, so issuing this early is always safe.
OSCAR_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

OSCAR_DEVICE void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

OSCAR_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

OSCAR_DEVICE float bf16_to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

OSCAR_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

OSCAR_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }
OSCAR_DEVICE float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// Round-to-nearest int8 with saturation (symmetric, [-127, 127]).
OSCAR_DEVICE int8_t quant_i8(float x, float inv_scale) {
  float q = rintf(x * inv_scale);
  q = fminf(fmaxf(q, -127.f), 127.f);
  return (int8_t)q;
}

}  // namespace oscar

#include <map>
#include <mutex>
#include <utility>
namespace oscar {
// cudaFuncSetAttribute acts on the current device only, so a process that drives
// several GPUs must raise a kernel's dynamic shared-memory limit on each of them.
// The (kernel, device) pairs already raised are remembered under a lock.
inline int ensure_smem_attr(const void* fn, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_pair(fn, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return 0;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return (int)e;
  done[key] = bytes;
  return 0;
}
template <class F>
inline int ensure_smem(F* fn, int bytes) {
  return ensure_smem_attr(reinterpret_cast<const void*>(fn), bytes);
}
}  // namespace oscar

#define OSCAR_RC(expr)          \
  do {                          \
    const int _rc = (expr);     \
    if (_rc) return _rc;        \
  } while (0)

#define OSCAR_CUDA_CHECK(expr)                                                   \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) return (int)_e;                                       \
  } while (0)
