// Gated DeltaNet prefill in chunk (WY) form on the tensor cores.
//
// For a chunk of C = 64 tokens starting from state S (dk x dv), with per-token
// decays g_t, G_t = sum_{u<=t} log g_u (cumulative inside the chunk), Gamma_t = e^{G_t}:
//
//     d   = U - W S                           (the delta-rule residuals d_t, C x dv)
//     O   = diag(Gamma) Q S + P d             (outputs before the gated RMSNorm)
//     S' = Gamma_last S + K^T diag(Gamma_last / Gamma) d
//
// with  A_ts = beta_t (Gamma_t / Gamma_s) k_t.k_s  (s < t),  T = (I + A)^-1,
//       W = T diag(beta Gamma) K,  U = T diag(beta) V,  P_ts = (Gamma_t / Gamma_s) q_t.k_s  (s <= t).
// This is the token recurrence S_t = g_t S_{t-1} + k_t d_t^T, d_t = beta_t (v_t - g_t S_{t-1}^T k_t),
// o_t = S_t^T q_t written for a whole chunk at once (same algebra as the per-token
// chunk form of gdn.cu; the reference serves this layer through its host framework's
// chunked gated-delta-rule operator).  Three kernels:
//
//   gdn_conv_kernel  one CTA per token: causal conv1d (kernel 4) + SiLU of every
//                    channel, L2 norms of q / k, beta and log g; writes bf16 q, k, v and
//                    the conv window of each request's last token;
//   gdn_wy_kernel    one CTA per (chunk, value head), fully parallel: K K^T and Q K^T
//                    (mma.sync), T by forward substitution in fp32, W and U^T (mma.sync);
//   gdn_scan_kernel  one CTA per (request, value head), sequential over the chunks:
//                    8 warps, each owning 16 value columns of S^T (fp32 accumulator
//                    fragments in registers for the whole request).  Per chunk
//                    X^T = S^T W^T, Y^T = S^T Q^T, d^T = U^T - X^T, O^T = Gamma Y^T + d^T P^T,
//                    S^T = Gamma_last S^T + (d^T diag(Gamma_last / Gamma)) K, then the gated
//                    RMSNorm over dv (partial sums across the 8 warps through shared memory).
//                    The next chunk's operands stream in with cp.async while this one runs.
//
// Operands are bf16 with fp32 accumulation; the state stays fp32 across the chunks
// of a step and is rounded to bf16 once when written back.
#include "common.cuh"
#include "mma.cuh"
#include "params.h"

namespace oscar {
namespace {

constexpr int kD = 128;   // dk == dv
constexpr int kCk = 64;   // chunk tokens

OSCAR_DEVICE bool is_long(const GdnParams& p, int req) {
  const int T = p.q_start[req + 1] - p.q_start[req];
  return p.long_min > 0 && T >= p.long_min && p.n_commit[req] == 0 && p.keep_pending[req] == 0;
}

// Byte offset of 16-byte chunk `c` of row `row` in a swizzled tile of `row_bytes`-byte
// rows (the chunk index is XOR-ed with the row's low three bits so that the eight
// rows an ldmatrix phase reads hit eight different bank groups).
OSCAR_DEVICE uint32_t swz(int row, int c, int row_bytes) { return row * row_bytes + ((c ^ (row & 7)) << 4); }

OSCAR_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill when the row does not exist
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
OSCAR_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
OSCAR_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

OSCAR_DEVICE uint32_t bf2_u32(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

OSCAR_DEVICE float softplusf(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// ------------------------------------------------------------------ conv + gates
// One CTA (256 threads) per (block of kConvTok consecutive tokens of one long request,
// slice of 256 16-byte channel chunks).  Each thread owns 8 channels and slides the
// 4-tap window over the block's tokens, so every qkvz row is read about once (plus a
// 3-row halo per block).  q / k chunks come first in channel order and a head's 16
// chunks sit in one half-warp: its L2 norm is a 16-lane butterfly per token.
constexpr int kConvThreads = 256;
constexpr int kConvTok = 16;

// Locates token block `bi` (kConvTok tokens) among the long requests.
OSCAR_DEVICE bool find_tok_block(const GdnParams& p, int bi, int& req, int& b) {
  for (int q = 0; q < p.R; ++q) {
    if (!is_long(p, q)) continue;
    const int n = (p.q_start[q + 1] - p.q_start[q] + kConvTok - 1) / kConvTok;
    if (bi < n) {
      req = q;
      b = bi;
      return true;
    }
    bi -= n;
  }
  return false;
}

__global__ void __launch_bounds__(kConvThreads) gdn_conv_kernel(GdnParams p) {
  int req, blk;
  if (!find_tok_block(p, blockIdx.x, req, blk)) return;
  const int t0 = p.q_start[req], T = p.q_start[req + 1] - t0;
  const int tb0 = blk * kConvTok, tb1 = min(T, tb0 + kConvTok);
  const int tid = threadIdx.x;
  const int r = p.Hv / p.Hk;
  const int Kd = p.Hk * kD;
  const int conv_dim = 2 * Kd + p.Hv * kD;
  const int n_qk = 2 * p.Hk * (kD / 8);  // q / k chunks
  const int n_chunks = conv_dim / 8;
  const int ck = blockIdx.y * kConvThreads + tid;  // this thread's channel chunk
  const long long grp = 2 * kD + 2 * r * kD;  // qkvz elements per key-head group
  const int slot = p.req_slot[req], par = p.parity[req];
  const __nv_bfloat16* cs = p.conv_state + ((long long)par * p.slots + slot) * conv_dim * 3;
  __nv_bfloat16* cs_out = p.conv_state + ((long long)(1 - par) * p.slots + slot) * conv_dim * 3;

  // gates of the block's tokens (first slice only)
  if (blockIdx.y == 0) {
    for (int idx = tid; idx < (tb1 - tb0) * p.Hv; idx += kConvThreads) {
      const int tok = t0 + tb0 + idx / p.Hv, h = idx % p.Hv;
      const int gk = h / r, hh = h % r;
      const __nv_bfloat16* barow = p.ba + (long long)tok * p.ld_ba + (long long)gk * 2 * r;
      const float bb = __bfloat162float(barow[hh]), aa = __bfloat162float(barow[r + hh]);
      p.ws_beta[(long long)tok * p.Hv + h] = sigmoidf_(bb);
      p.ws_lg[(long long)tok * p.Hv + h] = -__expf(p.A_log[h]) * softplusf(aa + p.dt_bias[h]);
    }
  }
  if (blockIdx.y * kConvThreads >= n_chunks) return;  // whole warps leave together (256 | slices)
  const bool active = ck < n_chunks;
  // channel chunk -> conv channel c0 and qkvz element offset
  int c0 = 0, head = 0;
  long long off = 0;
  bool isqk = false, isk = false;
  if (active) {
    if (ck < n_qk) {
      isqk = true;
      head = ck / (kD / 8);  // 0 .. 2 Hk - 1
      isk = head >= p.Hk;
      const int gk = isk ? head - p.Hk : head, seg = ck % (kD / 8);
      c0 = (isk ? Kd : 0) + gk * kD + 8 * seg;
      off = gk * grp + (isk ? kD : 0) + 8 * seg;
    } else {
      const int vc = ck - n_qk, h = vc / (kD / 8), seg = vc % (kD / 8);
      const int gk = h / r, hh = h % r;
      head = h;
      c0 = 2 * Kd + h * kD + 8 * seg;
      off = gk * grp + 2 * kD + (long long)hh * kD + 8 * seg;
    }
  }
  float w[8][4];
  float x0[8], x1[8], x2[8];  // raw inputs of tokens t-3, t-2, t-1
  if (active) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(p.conv_w) + (c0 + e));
      w[e][0] = w4.x;
      w[e][1] = w4.y;
      w[e][2] = w4.z;
      w[e][3] = w4.w;
    }
    auto load_raw = [&](int tt, float (&x)[8]) {
      if (tt >= 0) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.qkvz + (long long)(t0 + tt) * p.ld_qkvz + off));
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = __bfloat162float(h[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = __bfloat162float(cs[(long long)(c0 + e) * 3 + (3 + tt)]);
      }
    };
    load_raw(tb0 - 3, x0);
    load_raw(tb0 - 2, x1);
    load_raw(tb0 - 1, x2);
  }
  const float qscale = rsqrtf((float)kD);
  for (int t = tb0; t < tb1; ++t) {
    float y[8];
    float ss = 0.f;
    if (active) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.qkvz + (long long)(t0 + t) * p.ld_qkvz + off));
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xt = __bfloat162float(hb[e]);
        const float a = w[e][0] * x0[e] + w[e][1] * x1[e] + w[e][2] * x2[e] + w[e][3] * xt;
        y[e] = silu(a);
        ss += y[e] * y[e];
        x0[e] = x1[e];
        x1[e] = x2[e];
        x2[e] = xt;
      }
    }
    // L2 norm over the head's 16 chunks (half-warp); every lane takes part
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (!active) continue;
    const long long tok = t0 + t;
    uint4 o4;
    if (isqk) {
      const float sc = rsqrtf(ss + 1e-6f) * (isk ? 1.f : qscale);
      o4.x = bf2_u32(y[0] * sc, y[1] * sc);
      o4.y = bf2_u32(y[2] * sc, y[3] * sc);
      o4.z = bf2_u32(y[4] * sc, y[5] * sc);
      o4.w = bf2_u32(y[6] * sc, y[7] * sc);
      const int gk = isk ? head - p.Hk : head;
      *reinterpret_cast<uint4*>((isk ? p.ws_k : p.ws_q) + (tok * p.Hk + gk) * kD + (c0 % kD)) = o4;
    } else {
      o4.x = bf2_u32(y[0], y[1]);
      o4.y = bf2_u32(y[2], y[3]);
      o4.z = bf2_u32(y[4], y[5]);
      o4.w = bf2_u32(y[6], y[7]);
      *reinterpret_cast<uint4*>(p.ws_v + (tok * p.Hv + head) * kD + (c0 % kD)) = o4;
    }
  }
  // the conv window after the request's last token
  if (active && tb1 == T) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      cs_out[(long long)(c0 + e) * 3 + 0] = __float2bfloat16(x0[e]);
      cs_out[(long long)(c0 + e) * 3 + 1] = __float2bfloat16(x1[e]);
      cs_out[(long long)(c0 + e) * 3 + 2] = __float2bfloat16(x2[e]);
    }
  }
}

// Locates chunk `ci` among the long requests (in request order).  Returns false when
// there are fewer chunks.
OSCAR_DEVICE bool find_chunk(const GdnParams& p, int ci, int& req, int& c) {
  for (int q = 0; q < p.R; ++q) {
    if (!is_long(p, q)) continue;
    const int n = (p.q_start[q + 1] - p.q_start[q] + kCk - 1) / kCk;
    if (ci < n) {
      req = q;
      c = ci;
      return true;
    }
    ci -= n;
  }
  return false;
}

// Index of the first chunk of request `req` in the chunk workspaces.
OSCAR_DEVICE int chunk_base(const GdnParams& p, int req) {
  int base = 0;
  for (int q = 0; q < req; ++q)
    if (is_long(p, q)) base += (p.q_start[q + 1] - p.q_start[q] + kCk - 1) / kCk;
  return base;
}

// ------------------------------------------------------------------ WY representation
// One CTA (4 warps) per (chunk, value head).  Shared memory: K, Q, V tiles (64 x 128
// bf16, 256-byte swizzled rows), A (fp32 64 x 64), T diag(beta Gamma) and T diag(beta)
// (bf16 64 x 64, 128-byte swizzled rows), G and beta.
constexpr int kWyThreads = 128;
struct WyLayout {
  static constexpr int kK = 0, kQ = 16384, kV = 32768, kA = 49152, kTw = kA + 16384, kTu = kTw + 8192,
                       kG = kTu + 8192, kB = kG + 256, kTotal = kB + 256;
};

__global__ void __launch_bounds__(kWyThreads) gdn_wy_kernel(GdnParams p) {
  int req, c;
  if (!find_chunk(p, blockIdx.x, req, c)) return;
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sb = (uint32_t)__cvta_generic_to_shared(sm);
  float* Af = reinterpret_cast<float*>(sm + WyLayout::kA);
  float* Gs = reinterpret_cast<float*>(sm + WyLayout::kG);
  float* Bs = reinterpret_cast<float*>(sm + WyLayout::kB);
  const int h = blockIdx.y, r = p.Hv / p.Hk, gk = h / r;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, cq = lane & 3;
  const int t0 = p.q_start[req], T = p.q_start[req + 1] - t0;
  const int tok0 = t0 + c * kCk, n = min(kCk, T - c * kCk);
  const long long ci = (long long)chunk_base(p, req) + c;
  if (ci >= p.max_chunks) {
    if (tid == 0) record_status(p.status, kBadShape);
    return;
  }

  // ---- tiles (rows >= n zero-filled) and gates
  for (int v = tid; v < kCk * 16; v += kWyThreads) {
    const int t = v >> 4, ch = v & 15;
    const bool ok = t < n;
    const long long tk = ok ? tok0 + t : tok0;
    cp_async16(sb + WyLayout::kK + swz(t, ch, 256), p.ws_k + (tk * p.Hk + gk) * kD + 8 * ch, ok);
    cp_async16(sb + WyLayout::kQ + swz(t, ch, 256), p.ws_q + (tk * p.Hk + gk) * kD + 8 * ch, ok);
    cp_async16(sb + WyLayout::kV + swz(t, ch, 256), p.ws_v + (tk * p.Hv + h) * kD + 8 * ch, ok);
  }
  cp_async_commit();
  if (warp == 0) {
    // inclusive scan of log g over the chunk: lane owns tokens 2 lane, 2 lane + 1
    const int ta = 2 * lane, tb = ta + 1;
    const float la = ta < n ? p.ws_lg[(long long)(tok0 + ta) * p.Hv + h] : 0.f;
    const float lb = tb < n ? p.ws_lg[(long long)(tok0 + tb) * p.Hv + h] : 0.f;
    float s = la + lb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    Gs[tb] = s;
    Gs[ta] = s - lb;
    Bs[ta] = ta < n ? p.ws_beta[(long long)(tok0 + ta) * p.Hv + h] : 0.f;
    Bs[tb] = tb < n ? p.ws_beta[(long long)(tok0 + tb) * p.Hv + h] : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- K K^T and Q K^T for rows t in [16 warp, 16 warp + 16)
  {
    float kk[8][4], qk[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[i][e] = qk[i][e] = 0.f;
#pragma unroll
    for (int kt = 0; kt < 8; ++kt) {
      uint32_t ak[4], aq[4];
      const int ar = 16 * warp + (lane & 15), ac = 2 * kt + (lane >> 4);
      mma::ldsm_x4(sb + WyLayout::kK + swz(ar, ac, 256), ak[0], ak[1], ak[2], ak[3]);
      mma::ldsm_x4(sb + WyLayout::kQ + swz(ar, ac, 256), aq[0], aq[1], aq[2], aq[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int br = 16 * np + (lane & 7) + ((lane >> 4) << 3), bc = 2 * kt + ((lane >> 3) & 1);
        mma::ldsm_x4(sb + WyLayout::kK + swz(br, bc, 256), b0, b1, b2, b3);
        mma::mma_bf16(kk[2 * np], ak[0], ak[1], ak[2], ak[3], b0, b1);
        mma::mma_bf16(kk[2 * np + 1], ak[0], ak[1], ak[2], ak[3], b2, b3);
        mma::mma_bf16(qk[2 * np], aq[0], aq[1], aq[2], aq[3], b0, b1);
        mma::mma_bf16(qk[2 * np + 1], aq[0], aq[1], aq[2], aq[3], b2, b3);
      }
    }
    __nv_bfloat16* P = p.ws_p + (ci * p.Hv + h) * kCk * kCk;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int t = 16 * warp + g + 8 * hr, s0 = 8 * nt + 2 * cq;
        float av[2], pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int s = s0 + e;
          const float dec = __expf(Gs[t] - Gs[s]);
          av[e] = s < t ? Bs[t] * dec * kk[nt][2 * hr + e] : 0.f;
          pv[e] = s <= t ? dec * qk[nt][2 * hr + e] : 0.f;
        }
        *reinterpret_cast<float2*>(Af + t * kCk + s0) = make_float2(av[0], av[1]);
        *reinterpret_cast<uint32_t*>(P + t * kCk + s0) = bf2_u32(pv[0], pv[1]);
      }
    }
  }
  __syncthreads();

  // ---- T = (I + A)^-1 by forward substitution, column s per thread (fp32)
  if (tid < kCk) {
    const int s = tid;
    float x[kCk];
#pragma unroll
    for (int t = 0; t < kCk; ++t) {
      float acc = t == s ? 1.f : 0.f;
      const float* arow = Af + t * kCk;
#pragma unroll
      for (int u4 = 0; u4 < t / 4; ++u4) {
        const float4 a = *reinterpret_cast<const float4*>(arow + 4 * u4);
        acc = fmaf(-a.x, x[4 * u4], acc);
        acc = fmaf(-a.y, x[4 * u4 + 1], acc);
        acc = fmaf(-a.z, x[4 * u4 + 2], acc);
        acc = fmaf(-a.w, x[4 * u4 + 3], acc);
      }
#pragma unroll
      for (int u = (t / 4) * 4; u < t; ++u) acc = fmaf(-arow[u], x[u], acc);
      x[t] = acc;
    }
    const float bw = Bs[s] * __expf(Gs[s]), bu = Bs[s];
    uint8_t* tw = sm + WyLayout::kTw;
    uint8_t* tu = sm + WyLayout::kTu;
#pragma unroll
    for (int t = 0; t < kCk; ++t) {
      const uint32_t o = swz(t, s >> 3, 128) + (s & 7) * 2;
      *reinterpret_cast<__nv_bfloat16*>(tw + o) = __float2bfloat16(x[t] * bw);
      *reinterpret_cast<__nv_bfloat16*>(tu + o) = __float2bfloat16(x[t] * bu);
    }
  }
  if (tid < kCk) p.ws_g[(ci * p.Hv + h) * kCk + tid] = Gs[tid];
  __syncthreads();

  // ---- W = T diag(beta Gamma) K: rows t in [16 warp, +16), 128 columns
  {
    float acc[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a[4];
      mma::ldsm_x4(sb + WyLayout::kTw + swz(16 * warp + (lane & 15), 2 * ks + (lane >> 4), 128), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b0, b1, b2, b3;
        const int br = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), bc = 2 * np + (lane >> 4);
        mma::ldsm_x4_t(sb + WyLayout::kK + swz(br, bc, 256), b0, b1, b2, b3);
        mma::mma_bf16(acc[2 * np], a[0], a[1], a[2], a[3], b0, b1);
        mma::mma_bf16(acc[2 * np + 1], a[0], a[1], a[2], a[3], b2, b3);
      }
    }
    __nv_bfloat16* W = p.ws_w + (ci * p.Hv + h) * kCk * kD;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int t = 16 * warp + g + 8 * hr, d = 8 * nt + 2 * cq;
        *reinterpret_cast<uint32_t*>(W + t * kD + d) = bf2_u32(acc[nt][2 * hr], acc[nt][2 * hr + 1]);
      }
  }
  // ---- U^T = (diag(beta) V)^T T^T: dv rows [32 warp, +32), 64 token columns
  {
    float acc[2][8][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[m][i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int i = lane >> 3;
        const int ar = 16 * ks + (lane & 7) + ((i >> 1) << 3), ac = (32 * warp + 16 * m) / 8 + (i & 1);
        mma::ldsm_x4_t(sb + WyLayout::kV + swz(ar, ac, 256), a[m][0], a[m][1], a[m][2], a[m][3]);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int br = 16 * np + (lane & 7) + ((lane >> 4) << 3), bc = 2 * ks + ((lane >> 3) & 1);
        mma::ldsm_x4(sb + WyLayout::kTu + swz(br, bc, 128), b0, b1, b2, b3);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          mma::mma_bf16(acc[m][2 * np], a[m][0], a[m][1], a[m][2], a[m][3], b0, b1);
          mma::mma_bf16(acc[m][2 * np + 1], a[m][0], a[m][1], a[m][2], a[m][3], b2, b3);
        }
      }
    }
    __nv_bfloat16* Ut = p.ws_ut + (ci * p.Hv + h) * kD * kCk;
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int d = 32 * warp + 16 * m + g + 8 * hr, t = 8 * nt + 2 * cq;
          *reinterpret_cast<uint32_t*>(Ut + d * kCk + t) = bf2_u32(acc[m][nt][2 * hr], acc[m][nt][2 * hr + 1]);
        }
  }
}

// ------------------------------------------------------------------ sequential scan
// One CTA (8 warps) per (long request, value head).  Warp w owns value columns
// [16 w, 16 w + 16) of the state, kept transposed (S^T: 16 rows x 128 dk) as mma
// accumulator fragments.  Per chunk stage (bf16, swizzled rows): W [64][128],
// Q [64][128], K [64][128], U^T [128][64], P [64][64], z [64][128], G [64] fp32.
constexpr int kScanThreads = 256;
struct ScanLayout {
  static constexpr int kW = 0, kQ = 16384, kK = 32768, kU = 49152, kP = 65536, kZ = 73728, kG = 90112,
                       kStage = 90368, kRed = 2 * kStage, kTotal = kRed + 2 * 8 * 64 * 4;
};

__global__ void __launch_bounds__(kScanThreads, 1) gdn_scan_kernel(GdnParams p) {
  const int req = blockIdx.x, h = blockIdx.y;
  if (!is_long(p, req)) return;
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sb = (uint32_t)__cvta_generic_to_shared(sm);
  float* red = reinterpret_cast<float*>(sm + ScanLayout::kRed);  // [2][8 warps][64 tokens]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, cq = lane & 3;
  const int r = p.Hv / p.Hk, gk = h / r, hh = h % r;
  const int t0 = p.q_start[req], T = p.q_start[req + 1] - t0;
  const int nch = (T + kCk - 1) / kCk;
  const long long cbase = chunk_base(p, req);
  if (cbase + nch > p.max_chunks) {
    if (tid == 0) record_status(p.status, kBadShape);
    return;
  }
  const int slot = p.req_slot[req];
  __nv_bfloat16* st = p.state + ((long long)slot * p.Hv + h) * kD * kD;  // [dk][dv]
  const long long grp = 2 * kD + 2 * r * kD;
  const long long zoff = gk * grp + 2 * kD + (long long)r * kD + (long long)hh * kD;

  auto load_chunk = [&](int i) {
    const uint32_t s0 = sb + (i & 1) * ScanLayout::kStage;
    const int tok0 = t0 + i * kCk, n = min(kCk, T - i * kCk);
    const long long ci = cbase + i;
    const __nv_bfloat16* W = p.ws_w + (ci * p.Hv + h) * kCk * kD;
    const __nv_bfloat16* U = p.ws_ut + (ci * p.Hv + h) * kD * kCk;
    const __nv_bfloat16* P = p.ws_p + (ci * p.Hv + h) * kCk * kCk;
    for (int v = tid; v < kCk * 16; v += kScanThreads) {
      const int t = v >> 4, ch = v & 15;
      const bool ok = t < n;
      const long long tk = ok ? tok0 + t : tok0;
      cp_async16(s0 + ScanLayout::kW + swz(t, ch, 256), W + t * kD + 8 * ch, true);
      cp_async16(s0 + ScanLayout::kQ + swz(t, ch, 256), p.ws_q + (tk * p.Hk + gk) * kD + 8 * ch, ok);
      cp_async16(s0 + ScanLayout::kK + swz(t, ch, 256), p.ws_k + (tk * p.Hk + gk) * kD + 8 * ch, ok);
      cp_async16(s0 + ScanLayout::kZ + swz(t, ch, 256), p.qkvz + tk * p.ld_qkvz + zoff + 8 * ch, ok);
      const int d = v >> 3, uc = v & 7;  // U^T: 128 rows x 8 chunks
      cp_async16(s0 + ScanLayout::kU + swz(d, uc, 128), U + d * kCk + 8 * uc, true);
    }
    for (int v = tid; v < kCk * 8; v += kScanThreads) {
      const int t = v >> 3, ch = v & 7;
      cp_async16(s0 + ScanLayout::kP + swz(t, ch, 128), P + t * kCk + 8 * ch, true);
    }
    if (tid < 16) cp_async16(s0 + ScanLayout::kG + 16 * tid, p.ws_g + (ci * p.Hv + h) * kCk + 4 * tid, true);
    cp_async_commit();
  };

  load_chunk(0);
  // S^T fragments: rows dv = 16 warp + g (+8), columns dk = 8 nt + 2 cq (+1)
  float sT[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int dv = 16 * warp + g + 8 * (e >> 1), dk = 8 * nt + 2 * cq + (e & 1);
      sT[nt][e] = __bfloat162float(st[dk * kD + dv]);
    }
  const float nw0 = p.norm_w[16 * warp + g], nw1 = p.norm_w[16 * warp + g + 8];

  for (int i = 0; i < nch; ++i) {
    cp_async_wait<0>();
    __syncthreads();
    if (i + 1 < nch) load_chunk(i + 1);
    const uint32_t s0 = sb + (i & 1) * ScanLayout::kStage;
    const uint8_t* sp = sm + (i & 1) * ScanLayout::kStage;
    const float* Gs = reinterpret_cast<const float*>(sp + ScanLayout::kG);
    const int n = min(kCk, T - i * kCk);
    float X[8][4], Y[8][4];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) X[a][e] = Y[a][e] = 0.f;
    // ---- X^T = S^T W^T, Y^T = S^T Q^T  (16 x 64, K = 128)
#pragma unroll
    for (int kt = 0; kt < 8; ++kt) {
      const uint32_t a0 = bf2_u32(sT[2 * kt][0], sT[2 * kt][1]), a1 = bf2_u32(sT[2 * kt][2], sT[2 * kt][3]);
      const uint32_t a2 = bf2_u32(sT[2 * kt + 1][0], sT[2 * kt + 1][1]), a3 = bf2_u32(sT[2 * kt + 1][2], sT[2 * kt + 1][3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int br = 16 * np + (lane & 7) + ((lane >> 4) << 3), bc = 2 * kt + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        mma::ldsm_x4(s0 + ScanLayout::kW + swz(br, bc, 256), b0, b1, b2, b3);
        mma::mma_bf16(X[2 * np], a0, a1, a2, a3, b0, b1);
        mma::mma_bf16(X[2 * np + 1], a0, a1, a2, a3, b2, b3);
        mma::ldsm_x4(s0 + ScanLayout::kQ + swz(br, bc, 256), b0, b1, b2, b3);
        mma::mma_bf16(Y[2 * np], a0, a1, a2, a3, b0, b1);
        mma::mma_bf16(Y[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- d^T = U^T - X^T; Y^T scaled by Gamma_t
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int tc = 8 * nt + 2 * cq;
      const float ga = __expf(Gs[tc]), gb = __expf(Gs[tc + 1]);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int d = 16 * warp + g + 8 * hr;
        const uint32_t u = *reinterpret_cast<const uint32_t*>(sp + ScanLayout::kU + swz(d, nt, 128) + 4 * cq);
        const float2 uf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
        X[nt][2 * hr] = uf.x - X[nt][2 * hr];
        X[nt][2 * hr + 1] = uf.y - X[nt][2 * hr + 1];
        Y[nt][2 * hr] *= ga;
        Y[nt][2 * hr + 1] *= gb;
      }
    }
    // ---- O^T += d^T P^T (P lower triangular: k-tile ks contributes to token tiles >= it)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t a0 = bf2_u32(X[2 * ks][0], X[2 * ks][1]), a1 = bf2_u32(X[2 * ks][2], X[2 * ks][3]);
      const uint32_t a2 = bf2_u32(X[2 * ks + 1][0], X[2 * ks + 1][1]), a3 = bf2_u32(X[2 * ks + 1][2], X[2 * ks + 1][3]);
#pragma unroll
      for (int np = ks; np < 4; ++np) {
        const int br = 16 * np + (lane & 7) + ((lane >> 4) << 3), bc = 2 * ks + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        mma::ldsm_x4(s0 + ScanLayout::kP + swz(br, bc, 128), b0, b1, b2, b3);
        mma::mma_bf16(Y[2 * np], a0, a1, a2, a3, b0, b1);
        mma::mma_bf16(Y[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- gated RMSNorm over dv: per-token sums of squares across the 8 warps
    float* rb = red + (i & 1) * 8 * 64;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float s0v = Y[nt][0] * Y[nt][0] + Y[nt][2] * Y[nt][2];
      float s1v = Y[nt][1] * Y[nt][1] + Y[nt][3] * Y[nt][3];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        s0v += __shfl_xor_sync(0xffffffffu, s0v, o);
        s1v += __shfl_xor_sync(0xffffffffu, s1v, o);
      }
      if (g == 0) *reinterpret_cast<float2*>(rb + warp * 64 + 8 * nt + 2 * cq) = make_float2(s0v, s1v);
    }
    // ---- S^T = Gamma_last S^T + (d^T diag(Gamma_last / Gamma)) K   (16 x 128, K = 64 tokens)
    {
      const float gl = Gs[kCk - 1];
      const float gamma = __expf(gl);
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sT[nt][e] *= gamma;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int ta = 16 * ks + 2 * cq, tb = ta + 8;
        const float fa0 = __expf(gl - Gs[ta]), fa1 = __expf(gl - Gs[ta + 1]);
        const float fb0 = __expf(gl - Gs[tb]), fb1 = __expf(gl - Gs[tb + 1]);
        const uint32_t a0 = bf2_u32(X[2 * ks][0] * fa0, X[2 * ks][1] * fa1);
        const uint32_t a1 = bf2_u32(X[2 * ks][2] * fa0, X[2 * ks][3] * fa1);
        const uint32_t a2 = bf2_u32(X[2 * ks + 1][0] * fb0, X[2 * ks + 1][1] * fb1);
        const uint32_t a3 = bf2_u32(X[2 * ks + 1][2] * fb0, X[2 * ks + 1][3] * fb1);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          const int br = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), bc = 2 * np + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          mma::ldsm_x4_t(s0 + ScanLayout::kK + swz(br, bc, 256), b0, b1, b2, b3);
          mma::mma_bf16(sT[2 * np], a0, a1, a2, a3, b0, b1);
          mma::mma_bf16(sT[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp's sums of squares are in
    // ---- outputs: o = bf16(o * rstd) * w * silu(z)
    const int tok0 = t0 + i * kCk;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int t = 8 * nt + 2 * cq + e2;
        if (t >= n) continue;
        float ss = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) ss += rb[w * 64 + t];
        const float rs = rsqrtf(ss / (float)kD + p.eps);
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int d = 16 * warp + g + 8 * hr;
          const float z = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(
              sp + ScanLayout::kZ + swz(t, d >> 3, 256) + (d & 7) * 2));
          float o = __bfloat162float(__float2bfloat16(Y[nt][2 * hr + e2] * rs)) * (hr ? nw1 : nw0);
          o *= silu(z);
          p.out[(long long)(tok0 + t) * p.Hv * kD + h * kD + d] = __float2bfloat16(o);
        }
      }
    }
  }
  // ---- state back to bf16 [dk][dv]
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int dv = 16 * warp + g + 8 * (e >> 1), dk = 8 * nt + 2 * cq + (e & 1);
      st[dk * kD + dv] = __float2bfloat16(sT[nt][e]);
    }
}

}  // namespace
}  // namespace oscar

// Workspace bytes the chunked prefill path needs for `T` tokens in at most
// `max_chunks` 64-token chunks (five regions, 256-byte aligned).
extern "C" long long oscar_gdn_chunk_ws_bytes(int T, int Hk, int Hv, int max_chunks) {
  auto al = [](long long b) { return (b + 255) / 256 * 256; };
  const long long D = oscar::kD, C = oscar::kCk;
  return al(2LL * T * Hk * D * 2) + al((long long)T * Hv * D * 2) + al(2LL * T * Hv * 4) +
         al((long long)max_chunks * Hv * (C * D * 2 * 2 + C * C * 2 + C * 4));
}

// Chunked prefill for the long requests of a step (see the top of this file).  `ws`
// holds oscar_gdn_chunk_ws_bytes(T, ...) bytes; T is the number of token rows.
extern "C" int oscar_gdn_chunked(oscar::GdnParams* params, int T, void* ws, cudaStream_t stream) {
  using namespace oscar;
  GdnParams& p = *params;
  if (p.R <= 0 || T <= 0 || p.long_min <= 0) return 0;
  if (p.dk != kD || p.dv != kD) return -500;
  auto al = [](long long b) { return (b + 255) / 256 * 256; };
  uint8_t* w = reinterpret_cast<uint8_t*>(ws);
  p.ws_q = reinterpret_cast<__nv_bfloat16*>(w);
  p.ws_k = p.ws_q + (long long)T * p.Hk * kD;
  w += al(2LL * T * p.Hk * kD * 2);
  p.ws_v = reinterpret_cast<__nv_bfloat16*>(w);
  w += al((long long)T * p.Hv * kD * 2);
  p.ws_beta = reinterpret_cast<float*>(w);
  p.ws_lg = p.ws_beta + (long long)T * p.Hv;
  w += al(2LL * T * p.Hv * 4);
  const long long cH = (long long)p.max_chunks * p.Hv;
  p.ws_w = reinterpret_cast<__nv_bfloat16*>(w);
  p.ws_ut = p.ws_w + cH * kCk * kD;
  p.ws_p = p.ws_ut + cH * kCk * kD;
  p.ws_g = reinterpret_cast<float*>(p.ws_p + cH * kCk * kCk);
  OSCAR_RC(ensure_smem(gdn_wy_kernel, WyLayout::kTotal));
  OSCAR_RC(ensure_smem(gdn_scan_kernel, ScanLayout::kTotal));
  {
    const int conv_dim = 2 * p.Hk * kD + p.Hv * kD;
    const int slices = (conv_dim / 8 + kConvThreads - 1) / kConvThreads;
    gdn_conv_kernel<<<dim3(T / kConvTok + p.R, slices), kConvThreads, 0, stream>>>(p);
  }
  gdn_wy_kernel<<<dim3(p.max_chunks, p.Hv), kWyThreads, WyLayout::kTotal, stream>>>(p);
  gdn_scan_kernel<<<dim3(p.R, p.Hv), kScanThreads, ScanLayout::kTotal, stream>>>(p);
  return (int)cudaGetLastError();
}
