// Fused FULL-attention KV write: one launch per layer and step does
//
//   qkv (bf16, from the qkv GEMM)
//     -> per-head RMSNorm of q and k (zero-centred weights, x * (1 + w))
//     -> partial RoPE (rotate-half on the first rot_dim dims)
//     -> rotation q @ R_k, k @ R_k, v @ R_v on the tensor cores: the normalised rows
//        are exact in bf16 and R is split into bf16 hi + lo parts, so two bf16
//        MMAs with fp32 accumulation reproduce the fp32 product to ~2^-16
//     -> q_rot (fp16) and the unclipped rotated k/v of the current chunk (fp16)
//        for the attention kernel, and fp32 sink/recent staging writes
//     -> per-vector sort-threshold clip of k/v (kth largest |x|, warp radix select)
//     -> asymmetric INT2 quantisation (fp16-rounded scale/zero, round-half-up)
//     -> packed codes + fp16 meta written into the 128-token page of the slot.
//
// Numerics follow the reference write path (backend.py:129-189, format.py:51-110):
// true fp32 division, floor(q + 0.5), scale floor 2^-14, scale/zero rounded to
// fp16 before use.
//
// Two launches: kv_prep (one CTA per token: load, RMSNorm, RoPE -> bf16 rows in a
// scratch buffer) and kv_rotate (64-row tiles: rotation MMAs, then one warp per row
// for the fresh copy, the staging write and clip/quantise/page write).
#include "common.cuh"
#include "mma.cuh"
#include "params.h"

namespace oscar {


namespace {

constexpr int kPage = 128;
constexpr int kThreads = 256;

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
// codes_row: token-major code row (K, 16-byte chunks swizzled by tok), or nullptr with
// vt_words/tok set: V is stored
// dim-major ("transposed") - dim d of the page owns kPage/16 words, and token tok sits
// in word d * kPage/16 + tok/16 at bit 16*(tok&1) + 2*((tok&15)>>1).  Tokens of one
// step share words, so the 2-bit fields are cleared and set with atomic reductions.
__device__ void quantize_vector(float (&x)[8], int n, int clip_idx, int D, uint8_t* codes_row,
                                __half* scale_dst, __half* zero_dst, uint32_t* vt_words = nullptr, int tok = 0) {
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
  // lane owns elements lane*n .. lane*n+n-1 (n = 4 or 8).  Pool bit order: each
  // 32-bit word holds dims 16w..16w+15 with dim 16w+2m+e at bit 16e+2m; the lanes
  // sharing a word OR their parts together and the first of them stores it.
  uint32_t part = 0;
  const int tbit = 16 * (tok & 1) + 2 * ((tok & 15) >> 1);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if (e < n) {
      float q = floorf(__fadd_rn(__fdiv_rn(__fsub_rn(x[e], zf), sf), 0.5f));
      q = fminf(fmaxf(q, 0.f), 3.f);
      if (vt_words) {
        uint32_t* w = vt_words + (lane * n + e) * (kPage / 16) + (tok >> 4);
        atomicAnd(w, ~(3u << tbit));
        atomicOr(w, ((uint32_t)q) << tbit);
      } else {
        const int j = (lane * n + e) & 15;
        part |= ((uint32_t)q) << (16 * (j & 1) + 2 * (j >> 1));
      }
    }
  }
  if (!vt_words) {
    for (int o = 1; o < 16 / n; o <<= 1) part |= __shfl_xor_sync(0xffffffffu, part, o);
    if (((lane * n) & 15) == 0) {
      // 16-byte chunks of a K code row are XOR-swizzled by the token (tok >> 1), so that
      // the attention kernels' per-token row reads hit distinct shared-memory banks
      const int w = (lane * n) >> 4, nch = D / 64;
      const int sw = (((w >> 2) ^ ((tok >> 1) & (nch - 1))) << 2) | (w & 3);
      reinterpret_cast<uint32_t*>(codes_row)[sw] = part;
    }
  }
  if (lane == 0) {
    *scale_dst = sh;
    *zero_dst = zh;
  }
}

// ---------------------------------------------------------------------------- prep
// xbuf rows: region K = [T][Hq + Hk] (q heads then k heads, rotated by R_k),
//            region V = [T][Hk]      (rotated by R_v), after region K.
__global__ void __launch_bounds__(kThreads) kv_prep_kernel(StoreParams p) {
  extern __shared__ float xin[];  // [nh][D]
  const int D = p.D, Hq = p.Hq, Hk = p.Hk;
  const int nh = Hq + 2 * Hk;
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < p.n_owner; i += gridDim.x * kThreads)
    p.owner[p.owner_seat[i]] = p.owner_val[i];
  const int t = blockIdx.x;
  if (t >= p.T) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* row = p.qkv + (long long)t * p.ld_qkv;
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int d = idx % D, h = idx / D;
    float v;
    if (h < Hq) v = __bfloat162float(row[p.q_off + h * p.q_head_stride + d]);
    else if (h < Hq + Hk) v = __bfloat162float(row[p.k_off + (h - Hq) * D + d]);
    else v = __bfloat162float(row[p.v_off + (h - Hq - Hk) * D + d]);
    xin[h * D + d] = v;
  }
  __syncthreads();
  for (int h = warp; h < Hq + Hk; h += kThreads / 32) {
    float* x = xin + h * D;
    const float* w = h < Hq ? p.q_norm_w : p.k_norm_w;
    if (w) {
      float ss = 0.f;
      for (int d = lane; d < D; d += 32) ss += x[d] * x[d];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + p.eps);
      for (int d = lane; d < D; d += 32) x[d] = __bfloat162float(__float2bfloat16(x[d] * inv * (p.norm_offset + w[d])));
      __syncwarp();
    }
    if (p.rope_cos && p.rot_dim > 0) {
      const int half = p.rot_dim / 2;
      const int pos = p.positions[t];
      const float* cs = p.rope_cos + (long long)pos * half;
      const float* sn = p.rope_sin + (long long)pos * half;
      for (int j = lane; j < half; j += 32) {
        const float a = x[j], b = x[j + half];
        x[j] = __bfloat162float(__float2bfloat16(a * cs[j] - b * sn[j]));
        x[j + half] = __bfloat162float(__float2bfloat16(b * cs[j] + a * sn[j]));
      }
      __syncwarp();
    }
  }
  __syncthreads();
  __nv_bfloat16* xk = p.xbuf + (long long)t * (Hq + Hk) * D;
  __nv_bfloat16* xv = p.xbuf + ((long long)p.T * (Hq + Hk) + (long long)t * Hk) * D;
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int h = idx / D;
    const __nv_bfloat16 b = __float2bfloat16(xin[idx]);
    if (h < Hq + Hk) xk[idx] = b;
    else xv[idx - (Hq + Hk) * D] = b;
  }
}

// ---------------------------------------------------------------------------- rotate
// rows per rotation tile: 16 rows (one m16 MMA slice) per CTA, so that a decode step's
// few hundred rows spread over the SMs instead of queueing behind a handful of CTAs
constexpr int kRT = 16;
constexpr int kYStride = 264;    // fp32 row stride of the output tile (bank padding)

struct RotSmem {
  static constexpr int X = 0;                       // [kRT][256] bf16, swizzled
  static constexpr int R = kRT * 512;               // R^T chunk hi + lo: 2 x [256][64] bf16 (64 KB)
  static constexpr int Y = R;                       // output [kRT][264] fp32, aliases R after the MMAs
  static constexpr int Y_BYTES = kRT * kYStride * 4;
  static constexpr int TOTAL = R + (Y_BYTES > 65536 ? Y_BYTES : 65536);
};

OSCAR_DEVICE uint32_t rswz(int n, int chunk) {  // [256][64] bf16 tile: 128 B rows, 8 chunks
  return n * 128 + ((chunk ^ (n & 7)) << 4);
}

OSCAR_DEVICE void cp_async16(void* dst, const void* src, bool pred) {
  const uint32_t d = smem_u32(dst);
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
OSCAR_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 2) kv_rotate_kernel(StoreParams p, int n_k_tiles) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* xs = sm + RotSmem::X;
  uint8_t* rhi = sm + RotSmem::R;
  uint8_t* rlo = rhi + 256 * 128;
  float* ys = reinterpret_cast<float*>(sm + RotSmem::Y);
  const int D = p.D, Hq = p.Hq, Hk = p.Hk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool vreg = blockIdx.x >= n_k_tiles;
  const long long rows_k = (long long)p.T * (Hq + Hk);
  const long long rows_total = vreg ? (long long)p.T * Hk : rows_k;
  const long long r0 = (long long)(vreg ? blockIdx.x - n_k_tiles : blockIdx.x) * kRT;
  const __nv_bfloat16* xsrc = p.xbuf + (vreg ? rows_k * D : 0);
  const __nv_bfloat16* RT_hi = vreg ? p.RvT_hi : p.RkT_hi;
  const __nv_bfloat16* RT_lo = vreg ? p.RvT_lo : p.RkT_lo;
  const int nrows = (int)min((long long)kRT, rows_total - r0);

  // X tile (rows beyond the region are zero-filled)
  for (int idx = tid; idx < kRT * 32; idx += kThreads) {
    const int r = idx >> 5, ch = idx & 31;
    const bool ok = r < nrows;
    const __nv_bfloat16* src = xsrc + (ok ? (r0 + r) * D + ch * 8 : 0);
    cp_async16(xs + mma::swz(r, ch), src, ok);
  }
  cp_async_wait_all();
  __syncthreads();

  if (RT_hi) {
    const int wn = warp;  // the tile's 16 rows x a 32-column slice of the 256 outputs
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const uint32_t xa = smem_u32(xs), ha = smem_u32(rhi), la = smem_u32(rlo);
    for (int kc = 0; kc < 4; ++kc) {
      __syncthreads();
      for (int idx = tid; idx < 256 * 8; idx += kThreads) {
        const int n = idx >> 3, ch = idx & 7;
        cp_async16(rhi + rswz(n, ch), RT_hi + (long long)n * D + kc * 64 + ch * 8, true);
        cp_async16(rlo + rswz(n, ch), RT_lo + (long long)n * D + kc * 64 + ch * 8, true);
      }
      cp_async_wait_all();
      __syncthreads();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t a0, a1, a2, a3;
        mma::ldsm_x4(xa + mma::swz((lane & 7) + ((lane >> 3) & 1) * 8, kc * 8 + 2 * ks + (lane >> 4)), a0, a1, a2,
                     a3);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          const int n = wn * 32 + np * 16 + (lane & 7) + (lane >> 4) * 8;
          const int ch = 2 * ks + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          mma::ldsm_x4(ha + rswz(n, ch), b0, b1, b2, b3);
          mma::mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
          mma::mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
          mma::ldsm_x4(la + rswz(n, ch), b0, b1, b2, b3);
          mma::mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
          mma::mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();  // R chunk dead: the output tile aliases it
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = wn * 32 + j * 8 + 2 * (lane & 3);
      const int ra = lane >> 2;
      *reinterpret_cast<float2*>(ys + ra * kYStride + col) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(ys + (ra + 8) * kYStride + col) = make_float2(acc[j][2], acc[j][3]);
    }
  } else {  // identity rotation
    for (int idx = tid; idx < kRT * D; idx += kThreads) {
      const int r = idx / D, d = idx % D;
      const uint4 v = *reinterpret_cast<const uint4*>(xs + mma::swz(r, d / 8));
      ys[r * kYStride + d] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&v)[d % 8]);
    }
  }
  __syncthreads();

  // per row: q output, or fresh copy + staging + clip/quantise/page write
  const int n = D / 32;
  for (int r = warp; r < nrows; r += kThreads / 32) {
    const long long gr = r0 + r;
    int t, h;
    bool is_q = false, is_v = vreg;
    if (!vreg) {
      t = (int)(gr / (Hq + Hk));
      h = (int)(gr % (Hq + Hk));
      if (h < Hq) is_q = true;
      else h -= Hq;
    } else {
      t = (int)(gr / Hk);
      h = (int)(gr % Hk);
    }
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = e < n ? ys[r * kYStride + lane * n + e] : 0.f;
    if (is_q) {
      __half* qo = p.q_out + ((long long)t * Hq + h) * D + lane * n;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < n) qo[e] = __float2half_rn(x[e]);
      continue;
    }
    __half* fresh = (is_v ? p.v_fresh : p.k_fresh) + ((long long)t * Hk + h) * D + lane * n;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < n) fresh[e] = __float2half_rn(x[e]);
    if (p.stage_seat) {
      const int seat = p.stage_seat[t];
      if (seat >= 0) {
        if (is_v) {  // dim-major per row: [row][Hk][D][128]
          float* st = p.stage_v + ((long long)(seat / kPage) * Hk + h) * D * kPage + seat % kPage;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < n) st[(long long)(lane * n + e) * kPage] = x[e];
        } else {  // token-major: [row * 128 + off][Hk][D]
          float* st = p.stage_k + ((long long)seat * Hk + h) * D + lane * n;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < n) st[e] = x[e];
        }
      }
    }
    const int slot = p.slots[t];
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
    __half* meta = reinterpret_cast<__half*>(page + 2 * kPage * cb);
    if (is_v)
      quantize_vector(x, n, p.v_clip_idx, D, nullptr, meta + 2 * kPage + off, meta + 3 * kPage + off,
                      reinterpret_cast<uint32_t*>(page + kPage * cb), off);
    else
      quantize_vector(x, n, p.k_clip_idx, D, page + off * cb, meta + off, meta + kPage + off, nullptr, off);
  }
}

}  // namespace
}  // namespace oscar

extern "C" int oscar_kv_store(const oscar::StoreParams* params, cudaStream_t stream) {
  using namespace oscar;
  const StoreParams& p = *params;
  if (p.T <= 0 && p.n_owner <= 0) return 0;
  if (p.D != 256 && p.D != 128) return -200;
  if (!p.xbuf) return -202;
  if ((p.Rk && !p.RkT_hi) || (p.Rv && !p.RvT_hi)) return -203;  // tensor-core path needs the bf16 split
  const int nh = p.Hq + 2 * p.Hk;
  const size_t smem_prep = (size_t)nh * p.D * sizeof(float);
  if (smem_prep > 200 * 1024) return -201;
  OSCAR_RC(ensure_smem(kv_prep_kernel, 200 * 1024));
  OSCAR_RC(ensure_smem(kv_rotate_kernel, RotSmem::TOTAL));
  const int grid_prep = p.T > 0 ? p.T : 1;
  kv_prep_kernel<<<grid_prep, kThreads, smem_prep, stream>>>(p);
  if (p.T <= 0) return (int)cudaGetLastError();
  const long long rows_k = (long long)p.T * (p.Hq + p.Hk), rows_v = (long long)p.T * p.Hk;
  const int n_k = (int)((rows_k + kRT - 1) / kRT), n_v = (int)((rows_v + kRT - 1) / kRT);
  kv_rotate_kernel<<<n_k + n_v, kThreads, RotSmem::TOTAL, stream>>>(p, n_k);
  return (int)cudaGetLastError();
}
