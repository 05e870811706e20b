// Fused FULL-attention KV write: one launch per layer and step does
//
//   qkv (bf16, from the qkv GEMM)
//     -> per-head RMSNorm of q and k (zero-centred weights, x * (1 + w))
//     -> partial RoPE (rotate-half on the first rot_dim dims)
//     -> fp32 rotation q @ R_k, k @ R_k, v @ R_v
//     -> q_rot (fp16) and the unclipped rotated k/v of the current chunk (fp16)
//        for the attention kernel, and fp32 sink/recent staging writes
//     -> per-vector sort-threshold clip of k/v (kth largest |x|, warp radix select)
//     -> asymmetric INT2 quantisation (fp16-rounded scale/zero, round-half-up)
//     -> packed codes + fp16 meta written into the 128-token page of the slot.
//
// Numerics follow the reference write path (backend.py:129-189, format.py:51-110):
// true fp32 division, floor(q + 0.5), scale floor 2^-14, scale/zero rounded to
// fp16 before use.  Rotation is a plain fp32 dot product per output column.
#include "common.cuh"
#include "params.h"

namespace oscar {


namespace {

constexpr int kPage = 128;
constexpr int kThreads = 256;
constexpr int kAcc = 32;  // (token, head) rows rotated per pass over R

__device__ __forceinline__ float kth_largest_abs(const float (&x)[8], int n, int kth) {
  uint32_t a[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = e < n ? (__float_as_uint(x[e]) & 0x7fffffffu) : 0u;
  uint32_t prefix = 0;
  for (int b = 30; b >= 0; --b) {
    const uint32_t cand = prefix | (1u << b);
    int c = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) c += (e < n && a[e] >= cand) ? 1 : 0;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= kth) prefix = cand;
  }
  return __uint_as_float(prefix);
}

// One warp quantises one (token, head) vector of D = 32 * n elements.
__device__ void quantize_vector(float (&x)[8], int n, int clip_idx, int D, uint8_t* codes_row,
                                __half* scale_dst, __half* zero_dst) {
  const int lane = threadIdx.x & 31;
  if (clip_idx >= 0) {
    const float thr = kth_largest_abs(x, n, D - clip_idx);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < n) x[e] = fminf(fmaxf(x[e], -thr), thr);
  }
  float lo = INFINITY, hi = -INFINITY;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (e < n) {
      lo = fminf(lo, x[e]);
      hi = fmaxf(hi, x[e]);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  float scale = __fdiv_rn(__fsub_rn(hi, lo), 3.0f);
  const float floor_v = 6.103515625e-05f;  // 2^-14
  scale = scale > floor_v ? scale : floor_v;
  const __half sh = __float2half_rn(scale);
  const __half zh = __float2half_rn(lo);
  const float sf = __half2float(sh), zf = __half2float(zh);
  // lane owns elements lane*n .. lane*n+n-1 (n is a multiple of 4): n/4 bytes.
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if (e < n) {
      float q = floorf(__fadd_rn(__fdiv_rn(__fsub_rn(x[e], zf), sf), 0.5f));
      q = fminf(fmaxf(q, 0.f), 3.f);
      packed |= ((uint32_t)q) << (2 * e);
    }
  }
  if (n == 8) {
    reinterpret_cast<uint16_t*>(codes_row)[lane] = (uint16_t)packed;
  } else if (n == 4) {
    codes_row[lane] = (uint8_t)packed;
  }
  if (lane == 0) {
    *scale_dst = sh;
    *zero_dst = zh;
  }
}

template <int TT>
__global__ void __launch_bounds__(kThreads) kv_store_kernel(StoreParams p) {
  extern __shared__ float sm[];
  const int D = p.D;
  const int Hq = p.Hq, Hk = p.Hk;
  const int nh = Hq + 2 * Hk;  // q heads, k heads, v heads
  float* xin = sm;                    // [TT][nh][D]
  float* kvrot = sm + TT * nh * D;    // [TT][2*Hk][D]

  // Owner-tag updates of this step (identical for every layer; only the first
  // FULL layer's launch carries them).
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < p.n_owner; i += gridDim.x * kThreads)
    p.owner[p.owner_seat[i]] = p.owner_val[i];

  const int t0 = blockIdx.x * TT;
  const int ntok = min(TT, p.T - t0);
  if (ntok <= 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- load q/k/v rows (bf16 -> fp32) -------------------------------------------------
  for (int idx = tid; idx < ntok * nh * D; idx += kThreads) {
    const int d = idx % D;
    const int h = (idx / D) % nh;
    const int t = idx / (D * nh);
    const __nv_bfloat16* row = p.qkv + (long long)(t0 + t) * p.ld_qkv;
    float v;
    if (h < Hq) v = __bfloat162float(row[p.q_off + h * p.q_head_stride + d]);
    else if (h < Hq + Hk) v = __bfloat162float(row[p.k_off + (h - Hq) * D + d]);
    else v = __bfloat162float(row[p.v_off + (h - Hq - Hk) * D + d]);
    xin[(t * nh + h) * D + d] = v;
  }
  __syncthreads();

  // ---- per-head RMSNorm of q and k, then partial RoPE ---------------------------------
  // warp w handles rows w, w+8, ... of the (token, head) rows that need it.
  const int n_qk = Hq + Hk;
  for (int r = warp; r < ntok * n_qk; r += kThreads / 32) {
    const int t = r / n_qk, h = r % n_qk;
    float* x = xin + (t * nh + h) * D;
    const float* w = h < Hq ? p.q_norm_w : p.k_norm_w;
    if (w) {
      float ss = 0.f;
      for (int d = lane; d < D; d += 32) ss += x[d] * x[d];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + p.eps);
      for (int d = lane; d < D; d += 32) {
        // round through bf16 like the model's norm output
        x[d] = __bfloat162float(__float2bfloat16(x[d] * inv * (p.norm_offset + w[d])));
      }
      __syncwarp();
    }
    if (p.rope_cos && p.rot_dim > 0) {
      const int half = p.rot_dim / 2;
      const int pos = p.positions[t0 + t];
      const float* cs = p.rope_cos + (long long)pos * half;
      const float* sn = p.rope_sin + (long long)pos * half;
      for (int j = lane; j < half; j += 32) {
        const float a = x[j], b = x[j + half];
        const float c = cs[j], s = sn[j];
        x[j] = __bfloat162float(__float2bfloat16(a * c - b * s));
        x[j + half] = __bfloat162float(__float2bfloat16(b * c + a * s));
      }
      __syncwarp();
    }
  }
  __syncthreads();

  // ---- rotation: q and k rows by R_k, v rows by R_v -----------------------------------
  // Rows are processed in groups of kAcc; row index r enumerates (t, h).
  {
    // rows: first every (t, q/k head) by R_k, then every (t, v head) by R_v
    const int nk_rows = ntok * (Hq + Hk);
    const int nv_rows = ntok * Hk;
    for (int pass = 0; pass < 2; ++pass) {
      const float* R = pass == 0 ? p.Rk : p.Rv;
      const int nrows = pass == 0 ? nk_rows : nv_rows;
      for (int g0 = 0; g0 < nrows; g0 += kAcc) {
        const int nr = min(kAcc, nrows - g0);
        int base[kAcc];
        float acc[kAcc];
#pragma unroll
        for (int r = 0; r < kAcc; ++r) {
          const int rr = g0 + (r < nr ? r : 0);
          int t, h;
          if (pass == 0) { t = rr / (Hq + Hk); h = rr % (Hq + Hk); }
          else { t = rr / Hk; h = Hq + Hk + rr % Hk; }
          base[r] = (t * nh + h) * D;
          acc[r] = 0.f;
        }
        const int d = tid;
        if (d < D) {
          if (R) {
            for (int i = 0; i < D; ++i) {
              const float rv = __ldg(R + (long long)i * D + d);
#pragma unroll
              for (int r = 0; r < kAcc; ++r) acc[r] = fmaf(xin[base[r] + i], rv, acc[r]);
            }
          } else {
#pragma unroll
            for (int r = 0; r < kAcc; ++r) acc[r] = xin[base[r] + d];
          }
#pragma unroll
          for (int r = 0; r < kAcc; ++r) {
            if (r < nr) {
              const int rr = g0 + r;
              if (pass == 0) {
                const int t = rr / (Hq + Hk), h = rr % (Hq + Hk);
                if (h < Hq) p.q_out[((long long)(t0 + t) * Hq + h) * D + d] = __float2half_rn(acc[r]);
                else kvrot[(t * 2 * Hk + (h - Hq)) * D + d] = acc[r];
              } else {
                const int t = rr / Hk, h = rr % Hk;
                kvrot[(t * 2 * Hk + Hk + h) * D + d] = acc[r];
              }
            }
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- per (token, head) K and V vectors: fresh copy, staging, clip, quantise, page write
  const int n = D / 32;  // elements per lane (D in {128, 256} -> 4 or 8)
  for (int vidx = warp; vidx < ntok * 2 * Hk; vidx += kThreads / 32) {
    const int t = vidx / (2 * Hk), hh = vidx % (2 * Hk);
    const bool is_v = hh >= Hk;
    const int h = is_v ? hh - Hk : hh;
    const int tok = t0 + t;
    const float* src = kvrot + (t * 2 * Hk + hh) * D;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = e < n ? src[lane * n + e] : 0.f;
    // unclipped rotated values for the current chunk
    __half* fresh = (is_v ? p.v_fresh : p.k_fresh) + ((long long)tok * Hk + h) * D + lane * n;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < n) fresh[e] = __float2half_rn(x[e]);
    if (p.stage_seat) {
      const int seat = p.stage_seat[tok];
      if (seat >= 0) {
        float* st = (is_v ? p.stage_v : p.stage_k) + ((long long)seat * Hk + h) * D + lane * n;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < n) st[e] = x[e];
      }
    }
    const int slot = p.slots[tok];
    if (slot < 0) continue;
    const int blk = slot / kPage, off = slot % kPage;
    if (p.kv_mode == 1) {
      __nv_bfloat16* dst = (is_v ? p.vc : p.kc) + (((long long)blk * kPage + off) * Hk + h) * D + lane * n;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < n) dst[e] = __float2bfloat16(x[e]);
      continue;
    }
    uint8_t* page = p.pool + ((long long)blk * Hk + h) * p.page_bytes;
    const int cb = D / 4;
    uint8_t* codes = page + (is_v ? kPage * cb : 0) + off * cb;
    __half* meta = reinterpret_cast<__half*>(page + 2 * kPage * cb);
    __half* sdst = meta + (is_v ? 2 : 0) * kPage + off;
    __half* zdst = meta + (is_v ? 3 : 1) * kPage + off;
    quantize_vector(x, n, is_v ? p.v_clip_idx : p.k_clip_idx, D, codes, sdst, zdst);
  }
}

}  // namespace
}  // namespace oscar

extern "C" int oscar_kv_store(const oscar::StoreParams* params, cudaStream_t stream) {
  using namespace oscar;
  const StoreParams& p = *params;
  if (p.T <= 0 && p.n_owner <= 0) return 0;
  if (p.D % 32 || p.D > 256 || p.D < 128) return -200;
  const int nh = p.Hq + 2 * p.Hk;
  const bool wide = p.T >= 512;
  const int TT = wide ? 4 : 1;
  const size_t smem = (size_t)TT * (nh + 2 * p.Hk) * p.D * sizeof(float);
  if (smem > 220 * 1024) return -201;
  int grid = (p.T + TT - 1) / TT;
  if (grid < 1) grid = 1;
  if (wide) {
    static bool a4 = false;
    if (!a4) {
      OSCAR_CUDA_CHECK(cudaFuncSetAttribute(kv_store_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
      a4 = true;
    }
    kv_store_kernel<4><<<grid, kThreads, smem, stream>>>(p);
  } else {
    static bool a1 = false;
    if (!a1) {
      OSCAR_CUDA_CHECK(cudaFuncSetAttribute(kv_store_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
      a1 = true;
    }
    kv_store_kernel<1><<<grid, kThreads, smem, stream>>>(p);
  }
  return (int)cudaGetLastError();
}
