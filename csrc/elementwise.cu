// Memory-bound per-token kernels of the hybrid model.  Each one produces the
// int8 activation + per-token scale that the next W8A8 GEMM consumes, so no
// activation makes an extra round trip through HBM:
//
//   rmsnorm_quant   fp32 residual -> RMSNorm (x * (off + w)) -> bf16 rounding -> int8, scale
//   swiglu_quant    bf16 [gate | up] -> silu(gate) * up -> int8, scale
//   act_quant       bf16 -> int8, scale
//   embed           token ids -> fp32 residual rows (bf16 table)
//   argmax          per-row (value, index) of bf16 logits, vocab-parallel aware
#include "common.cuh"

namespace oscar {
namespace {

constexpr int kT = 256;  // threads per token-block

// Per-token symmetric int8 quantisation of `n` values held in registers.
template <int PER>
OSCAR_DEVICE void quant_store(const float (&v)[PER], int n_valid_base, int H, int8_t* out_row, float* scale_out,
                              float* red) {
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int i = n_valid_base + e * kT;
    if (i < H) amax = fmaxf(amax, fabsf(v[e]));
  }
  amax = block_max<kT / 32>(amax, red);
  const float inv = amax > 0.f ? 127.f / amax : 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int i = n_valid_base + e * kT;
    if (i < H) out_row[i] = quant_i8(v[e], inv);
  }
  if (threadIdx.x == 0) *scale_out = amax > 0.f ? amax / 127.f : 1.f;
}

template <int PER>
__global__ void __launch_bounds__(kT) rmsnorm_quant_kernel(float* __restrict__ x, long long ldx,
                                                         const float* __restrict__ delta, long long ldd,
                                                         const float* __restrict__ w, float off, float eps, int H,
                                                         int8_t* __restrict__ out, float* __restrict__ scale,
                                                         __nv_bfloat16* __restrict__ out_bf16) {
  __shared__ float red[kT / 32];
  const int t = blockIdx.x;
  float* xr = x + (long long)t * ldx;
  float v[PER];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int i = threadIdx.x + e * kT;
    v[e] = i < H ? xr[i] : 0.f;
    if (delta && i < H) {
      v[e] += delta[(long long)t * ldd + i];  // fused residual add
      xr[i] = v[e];
    }
    ss += v[e] * v[e];
  }
  ss = block_sum<kT / 32>(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int i = threadIdx.x + e * kT;
    if (i < H) {
      v[e] = __bfloat162float(__float2bfloat16(v[e] * inv * (off + w[i])));
      if (out_bf16) out_bf16[(long long)t * H + i] = __float2bfloat16(v[e]);
    }
  }
  if (out) quant_store<PER>(v, threadIdx.x, H, out + (long long)t * H, scale + t, red);
}

template <int PER>
__global__ void __launch_bounds__(kT) swiglu_quant_kernel(const __nv_bfloat16* __restrict__ gu, long long ld, int I,
                                                        int8_t* __restrict__ out, float* __restrict__ scale) {
  __shared__ float red[kT / 32];
  const int t = blockIdx.x;
  const __nv_bfloat16* r = gu + (long long)t * ld;
  float v[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int i = threadIdx.x + e * kT;
    if (i < I) {
      const float g = __bfloat162float(r[i]), u = __bfloat162float(r[I + i]);
      v[e] = __bfloat162float(__float2bfloat16(silu(g) * u));
    } else {
      v[e] = 0.f;
    }
  }
  quant_store<PER>(v, threadIdx.x, I, out + (long long)t * I, scale + t, red);
}

template <int PER>
__global__ void __launch_bounds__(kT) act_quant_kernel(const __nv_bfloat16* __restrict__ x, long long ld, int K,
                                                     int8_t* __restrict__ out, float* __restrict__ scale) {
  __shared__ float red[kT / 32];
  const int t = blockIdx.x;
  float v[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int i = threadIdx.x + e * kT;
    v[e] = i < K ? __bfloat162float(x[(long long)t * ld + i]) : 0.f;
  }
  quant_store<PER>(v, threadIdx.x, K, out + (long long)t * K, scale + t, red);
}

__global__ void embed_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ table, int H,
                             int vocab_begin, int vocab_end, float* __restrict__ out) {
  const int t = blockIdx.x;
  const int id = tok[t];
  const bool mine = id >= vocab_begin && id < vocab_end;
  const __nv_bfloat16* row = table + (long long)(id - vocab_begin) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[(long long)t * H + i] = mine ? __bfloat162float(row[i]) : 0.f;
}

// Row argmax with ties broken toward the lowest index (torch.argmax semantics).
__global__ void __launch_bounds__(kT) argmax_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int V,
                                                 int index_offset, float* __restrict__ best_val,
                                                 int* __restrict__ best_idx) {
  __shared__ float sv[kT / 32];
  __shared__ int si[kT / 32];
  const int t = blockIdx.x;
  const __nv_bfloat16* r = logits + (long long)t * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += kT) {
    const float x = __bfloat162float(r[i]);
    if (x > bv || (x == bv && i < bi)) {
      bv = x;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    bv = l < kT / 32 ? sv[l] : -INFINITY;
    bi = l < kT / 32 ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      best_val[t] = bv;
      best_idx[t] = bi + index_offset;
    }
  }
}

// fp32 residual rows -> bf16 (final hidden state for the lm_head / MTP head).
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, long long n, __nv_bfloat16* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16(x[i]);
}


}  // namespace
}  // namespace oscar

using namespace oscar;

#define OSCAR_PER_DISPATCH(H, CALL) \
  do {                              \
    const int per = ((H) + kT - 1) / kT; \
    if (per <= 4) { constexpr int PER = 4; CALL; } \
    else if (per <= 8) { constexpr int PER = 8; CALL; } \
    else if (per <= 16) { constexpr int PER = 16; CALL; } \
    else if (per <= 24) { constexpr int PER = 24; CALL; } \
    else if (per <= 40) { constexpr int PER = 40; CALL; } \
    else if (per <= 72) { constexpr int PER = 72; CALL; } \
    else return -400; \
  } while (0)

extern "C" int oscar_rmsnorm_quant(float* x, long long ldx, const float* delta, long long ldd, const float* w,
                                   float off, float eps, int T, int H, int8_t* out, float* scale,
                                   __nv_bfloat16* out_bf16, cudaStream_t s) {
  if (T <= 0) return 0;
  OSCAR_PER_DISPATCH(H, (rmsnorm_quant_kernel<PER><<<T, kT, 0, s>>>(x, ldx, delta, ldd, w, off, eps, H, out, scale, out_bf16)));
  return (int)cudaGetLastError();
}

extern "C" int oscar_swiglu_quant(const __nv_bfloat16* gu, long long ld, int T, int I, int8_t* out, float* scale,
                                  cudaStream_t s) {
  if (T <= 0) return 0;
  OSCAR_PER_DISPATCH(I, (swiglu_quant_kernel<PER><<<T, kT, 0, s>>>(gu, ld, I, out, scale)));
  return (int)cudaGetLastError();
}

extern "C" int oscar_act_quant(const __nv_bfloat16* x, long long ld, int T, int K, int8_t* out, float* scale,
                               cudaStream_t s) {
  if (T <= 0) return 0;
  OSCAR_PER_DISPATCH(K, (act_quant_kernel<PER><<<T, kT, 0, s>>>(x, ld, K, out, scale)));
  return (int)cudaGetLastError();
}

extern "C" int oscar_embed(const int* tok, const __nv_bfloat16* table, int T, int H, int vocab_begin, int vocab_end,
                           float* out, cudaStream_t s) {
  if (T <= 0) return 0;
  embed_kernel<<<T, 256, 0, s>>>(tok, table, H, vocab_begin, vocab_end, out);
  return (int)cudaGetLastError();
}

extern "C" int oscar_argmax(const __nv_bfloat16* logits, long long ld, int T, int V, int index_offset, float* best_val,
                            int* best_idx, cudaStream_t s) {
  if (T <= 0) return 0;
  argmax_kernel<<<T, kT, 0, s>>>(logits, ld, V, index_offset, best_val, best_idx);
  return (int)cudaGetLastError();
}

extern "C" int oscar_f32_to_bf16(const float* x, long long n, __nv_bfloat16* y, cudaStream_t s) {
  if (n <= 0) return 0;
  int grid = (int)((n + 255) / 256);
  if (grid > 4096) grid = 4096;
  f32_to_bf16_kernel<<<grid, 256, 0, s>>>(x, n, y);
  return (int)cudaGetLastError();
}
