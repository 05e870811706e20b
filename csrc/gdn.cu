// Gated DeltaNet (linear attention) layer core: causal conv1d (kernel 4) + SiLU,
// q/k L2 normalisation, gates beta = sigmoid(b), g = exp(-exp(A_log) * softplus(a + dt_bias)),
// the delta rule per value head
//
//     S_t = g_t S_{t-1} + k_t d_t^T,   d_t = beta_t (v_t - g_t S_{t-1}^T k_t),   o_t = S_t^T q_t / sqrt(dk)
//
// and the gated RMSNorm  o <- rmsnorm(o) * w * silu(z).
//
// Chunk form.  For a chunk of n tokens against the state S0 at its start, with
// G_t = prod_{u<=t} g_u:
//
//     d_t = beta_t (v_t - G_t S0^T k_t - sum_{s<t} (G_t/G_s)(k_s.k_t) d_s)
//     o_t = G_t S0^T q_t + sum_{s<=t} (G_t/G_s)(k_s.q_t) d_s
//     S_w = G_w S0 + sum_{s<=w} (G_w/G_s) k_s d_s^T
//
// so a chunk reads S0 once (two dot products per token and column), solves a
// small scalar triangular system per column and writes the state once.  One CTA
// per (request, value head); thread j owns column j.  The CTA first stages the
// whole 128 x 128 state in shared memory with coalesced 16-byte loads (bf16 for
// a single decode/verify chunk, fp32 when many chunks of a prefill update it in
// place), so the column loops never wait on global memory.
//
// Speculative decoding uses deferred commit instead of per-draft snapshots: a
// verify step computes outputs for all its tokens from the committed state and
// keeps their raw inputs as "pending"; it writes back only the state after the
// tokens accepted in the previous step (n_commit), which it replays first.
// Every step therefore reads and writes the recurrent state exactly once.
#include "common.cuh"
#include "params.h"

namespace oscar {


namespace {

constexpr int kD = 128;  // dk == dv
constexpr int kThreads = 256;  // two threads per state column (rows 0-63 / 64-127)
constexpr int kHalf = 64;

OSCAR_DEVICE float softplusf(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

template <int kC, bool kF32State>
__global__ void __launch_bounds__(kThreads) gdn_chunk_kernel(GdnParams p) {
  // staged state [dk][dv]: fp32 (kF32State, updated in place across chunks) or bf16
  extern __shared__ __align__(16) uint8_t s_raw[];
  float* sS = reinterpret_cast<float*>(s_raw);
  __nv_bfloat16* sSb = reinterpret_cast<__nv_bfloat16*>(s_raw);
  __shared__ __align__(16) float qT[kD][kC];  // normalised q / k, transposed: [dim][token]
  __shared__ __align__(16) float kT[kD][kC];
  __shared__ float KK[kC][kC], KQ[kC][kC];
  __shared__ float Lg[kC], Bt[kC];
  __shared__ float nrm[kC][2], red[kC][8];
  __shared__ float pb_b[16], pb_a[16];

  const int req = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = tid >> 1, hf = tid & 1, i0 = hf * kHalf;
  const int t0 = p.q_start[req], T = p.q_start[req + 1] - t0;
  const int a = p.n_commit[req];
  const int n_all = a + T;
  if (n_all <= 0) return;
  const bool keep = p.keep_pending[req] != 0;
  // long prefill requests run in the chunked tensor-core path (gdn_chunk.cu)
  if (p.long_min > 0 && T >= p.long_min && a == 0 && !keep) return;
  const int write_after = keep ? a - 1 : n_all - 1;  // last token included in the stored state
  const int slot = p.req_slot[req];
  const int r = p.Hv / p.Hk;
  const int gk = h / r, hh = h % r;
  const int Kd = p.Hk * p.dk;
  const int conv_dim = 2 * Kd + p.Hv * p.dv;
  const int cq = gk * p.dk + j, ck = Kd + gk * p.dk + j, cv = 2 * Kd + h * p.dv + j;
  const long long grp = (long long)gk * (2 * p.dk + 2 * r * p.dv);
  const int par = p.parity[req];
  const __nv_bfloat16* cs = p.conv_state + ((long long)par * p.slots + slot) * conv_dim * 3;
  __nv_bfloat16* cs_out = p.conv_state + ((long long)(1 - par) * p.slots + slot) * conv_dim * 3;
  const __nv_bfloat16* px = p.pend_x + ((long long)par * p.slots + slot) * p.P * conv_dim;
  __nv_bfloat16* px_out = p.pend_x + ((long long)(1 - par) * p.slots + slot) * p.P * conv_dim;
  __nv_bfloat16* pb = p.pend_ba + (long long)slot * p.P * 2 * p.Hv;
  __nv_bfloat16* st = p.state + ((long long)slot * p.Hv + h) * p.dk * p.dv;

  if (a > p.P || a > 16 || (keep && (n_all > kC || T > p.P))) {
    if (tid == 0) record_status(p.status, kBadShape);
    return;
  }
  // gate inputs of the tokens to commit, read before this CTA overwrites them
  if (tid < a) {
    pb_b[tid] = __bfloat162float(pb[tid * 2 * p.Hv + h]);
    pb_a[tid] = __bfloat162float(pb[tid * 2 * p.Hv + p.Hv + h]);
  }
  float wq[3], wk[3], wv[3], cwq[4], cwk[4], cwv[4];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    wq[i] = __bfloat162float(cs[cq * 3 + i]);
    wk[i] = __bfloat162float(cs[ck * 3 + i]);
    wv[i] = __bfloat162float(cs[cv * 3 + i]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    cwq[i] = p.conv_w[cq * 4 + i];
    cwk[i] = p.conv_w[ck * 4 + i];
    cwv[i] = p.conv_w[cv * 4 + i];
  }
  const float A = -__expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  const float qscale = rsqrtf((float)p.dk);
  const float nw = p.norm_w[j];

  // coalesced 16-byte staging of the state (dk * dv bf16 = 32 KB)
  {
    const uint4* src = reinterpret_cast<const uint4*>(st);
#pragma unroll 4
    for (int v = tid; v < kD * kD / 8; v += kThreads) {
      const uint4 w = __ldg(src + v);
      if (kF32State) {
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&w);
        float4* d = reinterpret_cast<float4*>(sS + v * 8);
        const float2 x0 = __bfloat1622float2(hb[0]), x1 = __bfloat1622float2(hb[1]);
        const float2 x2 = __bfloat1622float2(hb[2]), x3 = __bfloat1622float2(hb[3]);
        d[0] = make_float4(x0.x, x0.y, x1.x, x1.y);
        d[1] = make_float4(x2.x, x2.y, x3.x, x3.y);
      } else {
        reinterpret_cast<uint4*>(sSb)[v] = w;
      }
    }
  }
  __syncthreads();

  bool conv_saved = false;
  auto save_conv = [&]() {
    if (!hf) {
      if (hh == 0)
        for (int i = 0; i < 3; ++i) {
          cs_out[cq * 3 + i] = __float2bfloat16(wq[i]);
          cs_out[ck * 3 + i] = __float2bfloat16(wk[i]);
        }
      for (int i = 0; i < 3; ++i) cs_out[cv * 3 + i] = __float2bfloat16(wv[i]);
    }
    conv_saved = true;
  };
  if (keep && a == 0) save_conv();

  for (int c0 = 0; c0 < n_all; c0 += kC) {
    const int n = min(kC, n_all - c0);
    float vv[kC], zz[kC];
    // ---- conv + SiLU for every token of the chunk (channel j of q, k, v) ----
#pragma unroll
    for (int u = 0; u < kC; ++u) {
      vv[u] = zz[u] = 0.f;
      float qo = 0.f, ko = 0.f;
      if (u < n) {
        const int idx = c0 + u;
        float xq, xk, xv, braw, araw;
        if (idx < a) {
          const __nv_bfloat16* prow = px + (long long)idx * conv_dim;
          xq = __bfloat162float(prow[cq]);
          xk = __bfloat162float(prow[ck]);
          xv = __bfloat162float(prow[cv]);
          braw = pb_b[idx];
          araw = pb_a[idx];
        } else {
          const int t = idx - a;
          const __nv_bfloat16* row = p.qkvz + (long long)(t0 + t) * p.ld_qkvz + grp;
          const __nv_bfloat16* barow = p.ba + (long long)(t0 + t) * p.ld_ba + (long long)gk * 2 * r;
          const __nv_bfloat16 bq = row[j], bk = row[p.dk + j], bv = row[2 * p.dk + hh * p.dv + j];
          const __nv_bfloat16 bb = barow[hh], baa = barow[r + hh];
          xq = __bfloat162float(bq);
          xk = __bfloat162float(bk);
          xv = __bfloat162float(bv);
          braw = __bfloat162float(bb);
          araw = __bfloat162float(baa);
          zz[u] = __bfloat162float(row[2 * p.dk + r * p.dv + hh * p.dv + j]);
          if (keep && !hf) {
            __nv_bfloat16* pw = px_out + (long long)t * conv_dim;
            if (hh == 0) {
              pw[cq] = bq;
              pw[ck] = bk;
            }
            pw[cv] = bv;
            if (j == 0) {
              pb[t * 2 * p.Hv + h] = bb;
              pb[t * 2 * p.Hv + p.Hv + h] = baa;
            }
          }
        }
        float q = cwq[3] * xq, k = cwk[3] * xk, v = cwv[3] * xv;
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          q = fmaf(cwq[i], wq[i], q);
          k = fmaf(cwk[i], wk[i], k);
          v = fmaf(cwv[i], wv[i], v);
        }
        wq[0] = wq[1]; wq[1] = wq[2]; wq[2] = xq;
        wk[0] = wk[1]; wk[1] = wk[2]; wk[2] = xk;
        wv[0] = wv[1]; wv[1] = wv[2]; wv[2] = xv;
        if (keep && idx == a - 1) save_conv();
        qo = silu(q);
        ko = silu(k);
        vv[u] = silu(v);
        if (tid == 0) {
          Bt[u] = sigmoidf_(braw);
          Lg[u] = A * softplusf(araw + dtb);  // log g
        }
      }
      if (!hf) {
        qT[j][u] = qo;
        kT[j][u] = ko;
      }
    }
    __syncthreads();
    // ---- L2 norms of q and k per token (warp w: tokens w, w+8, ...) ----
    for (int u = warp; u < n; u += kThreads / 32) {
      float sq = 0.f, sk = 0.f;
      for (int i = lane; i < kD; i += 32) {
        sq += qT[i][u] * qT[i][u];
        sk += kT[i][u] * kT[i][u];
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      if (lane == 0) {
        nrm[u][0] = rsqrtf(sq + 1e-6f) * qscale;
        nrm[u][1] = rsqrtf(sk + 1e-6f);
      }
    }
    if (tid == 0)
      for (int u = 1; u < n; ++u) Lg[u] += Lg[u - 1];  // cumulative log decay
    __syncthreads();
    if (!hf) {
#pragma unroll
      for (int u = 0; u < kC; ++u) {
        qT[j][u] = u < n ? qT[j][u] * nrm[u][0] : 0.f;
        kT[j][u] = u < n ? kT[j][u] * nrm[u][1] : 0.f;
      }
    }
    __syncthreads();
    // ---- pairwise dot products k_s.k_t and k_s.q_t for s <= t ----
    for (int pr = warp; pr < n * n; pr += kThreads / 32) {
      const int s_ = pr / n, t_ = pr % n;
      if (s_ > t_) continue;
      float kk = 0.f, kq = 0.f;
      for (int i = lane; i < kD; i += 32) {
        kk += kT[i][s_] * kT[i][t_];
        kq += kT[i][s_] * qT[i][t_];
      }
      kk = warp_sum(kk);
      kq = warp_sum(kq);
      if (lane == 0) {
        KK[s_][t_] = kk;
        KQ[s_][t_] = kq;
      }
    }
    __syncthreads();
    // ---- pass 1: S0^T k_t and S0^T q_t for column j (rows i0 .. i0+63) ----
    float kvS[kC], qS[kC];
#pragma unroll
    for (int u = 0; u < kC; ++u) kvS[u] = qS[u] = 0.f;
#pragma unroll 2
    for (int i = i0; i < i0 + kHalf; ++i) {
      const float sv = kF32State ? sS[i * kD + j] : __bfloat162float(sSb[i * kD + j]);
#pragma unroll
      for (int u4 = 0; u4 < kC / 4; ++u4) {
        const float4 kk = *reinterpret_cast<const float4*>(&kT[i][4 * u4]);
        const float4 qq = *reinterpret_cast<const float4*>(&qT[i][4 * u4]);
        kvS[4 * u4] = fmaf(sv, kk.x, kvS[4 * u4]);
        kvS[4 * u4 + 1] = fmaf(sv, kk.y, kvS[4 * u4 + 1]);
        kvS[4 * u4 + 2] = fmaf(sv, kk.z, kvS[4 * u4 + 2]);
        kvS[4 * u4 + 3] = fmaf(sv, kk.w, kvS[4 * u4 + 3]);
        qS[4 * u4] = fmaf(sv, qq.x, qS[4 * u4]);
        qS[4 * u4 + 1] = fmaf(sv, qq.y, qS[4 * u4 + 1]);
        qS[4 * u4 + 2] = fmaf(sv, qq.z, qS[4 * u4 + 2]);
        qS[4 * u4 + 3] = fmaf(sv, qq.w, qS[4 * u4 + 3]);
      }
    }
#pragma unroll
    for (int u = 0; u < kC; ++u) {
      kvS[u] += __shfl_xor_sync(0xffffffffu, kvS[u], 1);
      qS[u] += __shfl_xor_sync(0xffffffffu, qS[u], 1);
    }
    // ---- triangular solve for d_t and the outputs o_t ----
    float dd[kC], ov[kC];
#pragma unroll
    for (int t = 0; t < kC; ++t) {
      dd[t] = 0.f;
      if (t < n) {
        float acc = vv[t] - __expf(Lg[t]) * kvS[t];
#pragma unroll
        for (int s_ = 0; s_ < kC; ++s_)
          if (s_ < t) acc -= __expf(Lg[t] - Lg[s_]) * KK[s_][t] * dd[s_];
        dd[t] = Bt[t] * acc;
      }
    }
#pragma unroll
    for (int u = 0; u < kC; ++u) {
      float o = 0.f;
      if (u < n && c0 + u >= a) {
        o = __expf(Lg[u]) * qS[u];
#pragma unroll
        for (int s_ = 0; s_ < kC; ++s_)
          if (s_ <= u) o += __expf(Lg[u] - Lg[s_]) * KQ[s_][u] * dd[s_];
      }
      ov[u] = o;
      const float ss = warp_sum(hf ? 0.f : o * o);
      if (lane == 0) red[u][warp] = ss;
    }
    __syncthreads();
    // ---- gated RMSNorm over dv and output ----
    if (!hf) {
#pragma unroll
      for (int u = 0; u < kC; ++u) {
        if (u < n && c0 + u >= a) {
          float ss = 0.f;
#pragma unroll
          for (int w = 0; w < kThreads / 32; ++w) ss += red[u][w];
          float o = ov[u] * rsqrtf(ss / (float)p.dv + p.eps);
          o = __bfloat162float(__float2bfloat16(o)) * nw;
          o = o * silu(zz[u]);
          p.out[(long long)(t0 + c0 + u - a) * p.Hv * p.dv + h * p.dv + j] = __float2bfloat16(o);
        }
      }
    }
    // ---- pass 2: state after token w of this chunk ----
    const int w = min(n - 1, write_after - c0);
    if (w >= 0) {
      const float Gw = __expf(Lg[w]);
      float cf[kC];
#pragma unroll
      for (int s_ = 0; s_ < kC; ++s_) cf[s_] = (s_ <= w) ? __expf(Lg[w] - Lg[s_]) * dd[s_] : 0.f;
#pragma unroll 2
      for (int i = i0; i < i0 + kHalf; ++i) {
        float v = Gw * (kF32State ? sS[i * kD + j] : __bfloat162float(sSb[i * kD + j]));
#pragma unroll
        for (int u4 = 0; u4 < kC / 4; ++u4) {
          const float4 kk = *reinterpret_cast<const float4*>(&kT[i][4 * u4]);
          v = fmaf(kk.x, cf[4 * u4], v);
          v = fmaf(kk.y, cf[4 * u4 + 1], v);
          v = fmaf(kk.z, cf[4 * u4 + 2], v);
          v = fmaf(kk.w, cf[4 * u4 + 3], v);
        }
        if (kF32State) {
          sS[i * kD + j] = v;
        } else {
          const __nv_bfloat16 bv = __float2bfloat16(v);
          st[i * p.dv + j] = bv;
          sSb[i * kD + j] = bv;  // a following chunk (non-speculative, > kC tokens) reads it
        }
      }
    }
    __syncthreads();
    if (write_after < c0 + n) break;  // the stored state ends inside this chunk
  }
  if (kF32State) {
    __syncthreads();
    for (int v = tid; v < kD * kD / 2; v += kThreads) {
      const float2 f = reinterpret_cast<const float2*>(sS)[v];
      reinterpret_cast<__nv_bfloat162*>(st)[v] = __floats2bfloat162_rn(f.x, f.y);
    }
  }
  if (!conv_saved) save_conv();
}

// ---------------------------------------------------------------------------
// Decode / MTP-verify variant (<= 8 tokens per request and value head, 4 warps).
// Same algebra as above with the two products on the tensor cores:
//   pass 1:  [k_1..k_8 ; q_1..q_8] (16 x dk) . S0 (dk x dv)   -> S0^T k_t, S0^T q_t
//   pass 2:  S_w = G_w S0 + [k_1..k_8] (dk x 8) . C (8 x dv),  C_s = (G_w / G_s) d_s
// (mma.sync m16n8k16, bf16 in, fp32 accumulate).  The state lives in shared memory
// as bf16 in an XOR-swizzled layout and crosses global memory once each way with
// 16-byte accesses; thread j owns value column j for the per-column recurrence.
constexpr int kDecC = 8;
constexpr int kDecThreads = 128;

OSCAR_DEVICE uint32_t sw16(int row, int chunk) {  // [row][128 bf16]: 16 chunks of 16 B per row
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}
OSCAR_DEVICE void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
OSCAR_DEVICE void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
OSCAR_DEVICE void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Optional per-CTA phase timeline of the decode kernel (globaltimer ns, 16 slots per CTA,
// thread 0); off unless a buffer was installed with oscar_gdn_trace.
__device__ unsigned long long* g_gdn_trace = nullptr;
OSCAR_DEVICE void gdn_mark(unsigned long long* t, int ev) {
  if (t != nullptr && threadIdx.x == 0)
    t[((long long)blockIdx.y * gridDim.x + blockIdx.x) * 16 + ev] = globaltimer_ns();
}

__global__ void __launch_bounds__(kDecThreads) gdn_decode_kernel(GdnParams p) {
  __shared__ __align__(128) uint8_t sS[kD * 256];   // state, bf16 [dk][dv] swizzled
  __shared__ __align__(128) uint8_t sA[16 * 256];   // rows 0-7: k_t, 8-15: q_t (bf16 [tok][dk])
  // one region, three lives: normalised k/q columns (fp32) -> pass-1 result -> pass-2 B operand
  __shared__ __align__(128) uint8_t sU[2 * kD * (kDecC + 1) * 4];
  float (*kT)[kDecC + 1] = reinterpret_cast<float (*)[kDecC + 1]>(sU);
  float (*qT)[kDecC + 1] = reinterpret_cast<float (*)[kDecC + 1]>(sU + kD * (kDecC + 1) * 4);
  float (*kvq)[kD] = reinterpret_cast<float (*)[kD]>(sU);  // rows t: S^T k_t, 8 + t: S^T q_t
  uint8_t* sC = sU;                                        // rows 0-7: C_s (bf16 [s][dv]), 8-15 zero
  __shared__ float KK[kDecC][kDecC], KQ[kDecC][kDecC];
  __shared__ float Lg[kDecC], Bt[kDecC];
  __shared__ float red[kDecC][2][4];

  unsigned long long* const tr = g_gdn_trace;
  gdn_mark(tr, 0);
  const int req = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = tid;
  const int t0 = p.q_start[req], T = p.q_start[req + 1] - t0;
  const int a = p.n_commit[req];
  const int n = a + T;
  if (n <= 0) return;
  const bool keep = p.keep_pending[req] != 0;
  const int w_last = keep ? a - 1 : n - 1;  // last token included in the stored state
  const int slot = p.req_slot[req];
  const int r = p.Hv / p.Hk;
  const int gk = h / r, hh = h % r;
  const int Kd = p.Hk * p.dk;
  const int conv_dim = 2 * Kd + p.Hv * p.dv;
  const int cq = gk * p.dk + j, ck = Kd + gk * p.dk + j, cv = 2 * Kd + h * p.dv + j;
  const long long grp = (long long)gk * (2 * p.dk + 2 * r * p.dv);
  const int par = p.parity[req];
  const __nv_bfloat16* cs = p.conv_state + ((long long)par * p.slots + slot) * conv_dim * 3;
  __nv_bfloat16* cs_out = p.conv_state + ((long long)(1 - par) * p.slots + slot) * conv_dim * 3;
  const __nv_bfloat16* px = p.pend_x + ((long long)par * p.slots + slot) * p.P * conv_dim;
  __nv_bfloat16* px_out = p.pend_x + ((long long)(1 - par) * p.slots + slot) * p.P * conv_dim;
  __nv_bfloat16* pb = p.pend_ba + (long long)slot * p.P * 2 * p.Hv;
  __nv_bfloat16* st = p.state + ((long long)slot * p.Hv + h) * p.dk * p.dv;
  if (n > kDecC || a > p.P || (keep && T > p.P)) {
    if (tid == 0) record_status(p.status, kBadShape);
    return;
  }
  const uint32_t sS_a = smem_u32(sS), sA_a = smem_u32(sA), sC_a = smem_u32(sC);

  // ---- raw inputs of every token of the chunk, issued as independent loads (one
  // memory latency for the chunk instead of one per token): pending tokens come from
  // the kept raw inputs, new tokens from the projection output.  Only thread 0 reads
  // the b / a gate inputs; it is also the only writer of this head's pending b / a,
  // after its reads.
  __nv_bfloat16 rq[kDecC], rk[kDecC], rv[kDecC], rz[kDecC], rb[kDecC], ra[kDecC];
  const __nv_bfloat16 bzero = __float2bfloat16(0.f);
#pragma unroll
  for (int u = 0; u < kDecC; ++u) {
    rq[u] = rk[u] = rv[u] = rz[u] = rb[u] = ra[u] = bzero;
    const int t = u - a;
    if (u < a) {
      const __nv_bfloat16* prow = px + (long long)u * conv_dim;
      rq[u] = prow[cq];
      rk[u] = prow[ck];
      rv[u] = prow[cv];
      if (tid == 0) {
        rb[u] = pb[u * 2 * p.Hv + h];
        ra[u] = pb[u * 2 * p.Hv + p.Hv + h];
      }
    } else if (u < n) {
      const __nv_bfloat16* row = p.qkvz + (long long)(t0 + t) * p.ld_qkvz + grp;
      rq[u] = row[j];
      rk[u] = row[p.dk + j];
      rv[u] = row[2 * p.dk + hh * p.dv + j];
      rz[u] = row[2 * p.dk + r * p.dv + hh * p.dv + j];
      if (tid == 0) {
        const __nv_bfloat16* barow = p.ba + (long long)(t0 + t) * p.ld_ba + (long long)gk * 2 * r;
        rb[u] = barow[hh];
        ra[u] = barow[r + hh];
      }
    }
  }
  float wq[3], wk[3], wv[3], cwq[4], cwk[4], cwv[4];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    wq[i] = __bfloat162float(cs[cq * 3 + i]);
    wk[i] = __bfloat162float(cs[ck * 3 + i]);
    wv[i] = __bfloat162float(cs[cv * 3 + i]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    cwq[i] = p.conv_w[cq * 4 + i];
    cwk[i] = p.conv_w[ck * 4 + i];
    cwv[i] = p.conv_w[cv * 4 + i];
  }
  // state -> shared memory with asynchronous 16-byte copies (swizzled chunks), issued
  // after the chunk's input loads so that those are not queued behind 32 KB; they
  // stream in while the conv / gate / norm work below runs
  {
    const uint4* src = reinterpret_cast<const uint4*>(st);
#pragma unroll
    for (int v = tid; v < kD * 16; v += kDecThreads) {
      const int row = v >> 4, ch = v & 15;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sS_a + sw16(row, ch)), "l"(src + v) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const float A = -__expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  // new tokens' raw inputs are kept pending for the next step
  if (keep) {
#pragma unroll
    for (int u = 0; u < kDecC; ++u) {
      if (u >= a && u < n) {
        const int t = u - a;
        __nv_bfloat16* pw = px_out + (long long)t * conv_dim;
        if (hh == 0) {
          pw[cq] = rq[u];
          pw[ck] = rk[u];
        }
        pw[cv] = rv[u];
        if (tid == 0) {
          pb[t * 2 * p.Hv + h] = rb[u];
          pb[t * 2 * p.Hv + p.Hv + h] = ra[u];
        }
      }
    }
  }

  // ---- conv + SiLU of channel j for every token ----
  auto save_conv = [&]() {
    if (hh == 0)
      for (int i = 0; i < 3; ++i) {
        cs_out[cq * 3 + i] = __float2bfloat16(wq[i]);
        cs_out[ck * 3 + i] = __float2bfloat16(wk[i]);
      }
    for (int i = 0; i < 3; ++i) cs_out[cv * 3 + i] = __float2bfloat16(wv[i]);
  };
  bool conv_saved = false;
  if (keep && a == 0) {
    save_conv();
    conv_saved = true;
  }
  float vv[kDecC], zz[kDecC], qv[kDecC], kv[kDecC];
  float sq_part[kDecC], sk_part[kDecC];
#pragma unroll
  for (int u = 0; u < kDecC; ++u) {
    vv[u] = qv[u] = kv[u] = 0.f;
    zz[u] = __bfloat162float(rz[u]);
    if (u < n) {
      const float xq = __bfloat162float(rq[u]), xk = __bfloat162float(rk[u]), xv = __bfloat162float(rv[u]);
      float q = cwq[3] * xq, k = cwk[3] * xk, v = cwv[3] * xv;
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        q = fmaf(cwq[i], wq[i], q);
        k = fmaf(cwk[i], wk[i], k);
        v = fmaf(cwv[i], wv[i], v);
      }
      wq[0] = wq[1]; wq[1] = wq[2]; wq[2] = xq;
      wk[0] = wk[1]; wk[1] = wk[2]; wk[2] = xk;
      wv[0] = wv[1]; wv[1] = wv[2]; wv[2] = xv;
      if (keep && u == a - 1) {
        save_conv();
        conv_saved = true;
      }
      qv[u] = silu(q);
      kv[u] = silu(k);
      vv[u] = silu(v);
      if (tid == 0) {
        Bt[u] = sigmoidf_(__bfloat162float(rb[u]));
        Lg[u] = A * softplusf(__bfloat162float(ra[u]) + dtb);
      }
    }
    sq_part[u] = warp_sum(qv[u] * qv[u]);
    sk_part[u] = warp_sum(kv[u] * kv[u]);
  }
  if (!conv_saved) save_conv();
  if (lane == 0)
#pragma unroll
    for (int u = 0; u < kDecC; ++u) {
      red[u][0][warp] = sq_part[u];
      red[u][1][warp] = sk_part[u];
    }
  __syncthreads();
  gdn_mark(tr, 1);
  // ---- L2-normalised q (times 1/sqrt(dk)) and k: fp32 columns and bf16 MMA rows ----
  const float qscale = rsqrtf((float)p.dk);
#pragma unroll
  for (int u = 0; u < kDecC; ++u) {
    const float sq = red[u][0][0] + red[u][0][1] + red[u][0][2] + red[u][0][3];
    const float sk = red[u][1][0] + red[u][1][1] + red[u][1][2] + red[u][1][3];
    const float qn = u < n ? qv[u] * rsqrtf(sq + 1e-6f) * qscale : 0.f;
    const float kn = u < n ? kv[u] * rsqrtf(sk + 1e-6f) : 0.f;
    qT[j][u] = qn;
    kT[j][u] = kn;
    *reinterpret_cast<__nv_bfloat16*>(sA + sw16(u, j >> 3) + (j & 7) * 2) = __float2bfloat16(kn);
    *reinterpret_cast<__nv_bfloat16*>(sA + sw16(8 + u, j >> 3) + (j & 7) * 2) = __float2bfloat16(qn);
  }
  if (tid == 0)
    for (int u = 1; u < n; ++u) Lg[u] += Lg[u - 1];  // cumulative log decay
  __syncthreads();
  gdn_mark(tr, 2);
  // ---- pairwise (G_t / G_s) k_s.k_t and (G_t / G_s) k_s.q_t (fp32): pair (s, t) on two
  // adjacent lanes, each summing half of the dims, decay factor folded in ----
  {
    const int pr = tid >> 1, half = tid & 1;
    const int s_ = pr >> 3, t_ = pr & 7;
    const bool live = s_ <= t_ && t_ < n;
    float kk = 0.f, kq = 0.f;
    if (live) {
#pragma unroll 8
      for (int i = half * 64; i < half * 64 + 64; ++i) {
        const float ks = kT[i][s_];
        kk = fmaf(ks, kT[i][t_], kk);
        kq = fmaf(ks, qT[i][t_], kq);
      }
    }
    kk += __shfl_xor_sync(0xffffffffu, kk, 1);
    kq += __shfl_xor_sync(0xffffffffu, kq, 1);
    if (live && half == 0) {
      const float e = __expf(Lg[t_] - Lg[s_]);
      KK[s_][t_] = e * kk;
      KQ[s_][t_] = e * kq;
    }
  }
  // the state copies have landed (this thread's), and every thread's (barrier)
  gdn_mark(tr, 3);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  gdn_mark(tr, 4);
  // ---- pass 1 (tensor cores): rows 0-7 S0^T k_t, rows 8-15 S0^T q_t; warp w: columns 32w.. ----
  {
    float acc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm4(sA_a + sw16(lane & 15, 2 * ks + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        uint32_t b0, b1, b2, b3;
        const int krow = 16 * ks + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm4t(sS_a + sw16(krow, (32 * warp + 16 * pr) / 8 + (lane >> 4)), b0, b1, b2, b3);
        mma_bf16_16816(acc[2 * pr], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(acc[2 * pr + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with the k/q columns that kvq overwrites
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = 32 * warp + 8 * nt + 2 * (lane & 3);
      *reinterpret_cast<float2*>(&kvq[lane >> 2][col]) = make_float2(acc[nt][0], acc[nt][1]);
      *reinterpret_cast<float2*>(&kvq[(lane >> 2) + 8][col]) = make_float2(acc[nt][2], acc[nt][3]);
    }
  }
  __syncthreads();
  gdn_mark(tr, 5);
  // ---- per column: triangular solve for d_t, outputs o_t ----
  float dd[kDecC], ov[kDecC];
#pragma unroll
  for (int t = 0; t < kDecC; ++t) {
    dd[t] = 0.f;
    if (t < n) {
      float acc = vv[t] - __expf(Lg[t]) * kvq[t][j];
#pragma unroll
      for (int s_ = 0; s_ < kDecC; ++s_)
        if (s_ < t) acc = fmaf(-KK[s_][t], dd[s_], acc);  // KK holds (G_t / G_s) k_s.k_t
      dd[t] = Bt[t] * acc;
    }
  }
  float os[kDecC];
#pragma unroll
  for (int u = 0; u < kDecC; ++u) {
    float o = 0.f;
    if (u < n && u >= a) {
      o = __expf(Lg[u]) * kvq[8 + u][j];
#pragma unroll
      for (int s_ = 0; s_ < kDecC; ++s_)
        if (s_ <= u) o = fmaf(KQ[s_][u], dd[s_], o);  // KQ holds (G_u / G_s) k_s.q_u
    }
    ov[u] = o;
    os[u] = warp_sum(o * o);
  }
  // C_s = (G_w / G_s) d_s as the B operand of pass 2 (rows 8-15 stay zero)
  const int w = w_last;
  float Gw = 0.f;
  __syncthreads();  // every column has read its pass-1 values: sC may overwrite them
  if (w >= 0) {
    Gw = __expf(Lg[w]);
#pragma unroll
    for (int s_ = 0; s_ < 16; ++s_) {
      const float c = (s_ < kDecC && s_ <= w) ? __expf(Lg[w] - Lg[s_]) * dd[s_ < kDecC ? s_ : 0] : 0.f;
      *reinterpret_cast<__nv_bfloat16*>(sC + sw16(s_, j >> 3) + (j & 7) * 2) = __float2bfloat16(c);
    }
  }
  __syncthreads();  // red (pass 1 values consumed) may be reused; sC complete
  gdn_mark(tr, 6);
  if (lane == 0)
#pragma unroll
    for (int u = 0; u < kDecC; ++u) red[u][0][warp] = os[u];
  __syncthreads();
  // ---- gated RMSNorm over dv and output ----
  const float nw = p.norm_w[j];
#pragma unroll
  for (int u = 0; u < kDecC; ++u) {
    if (u < n && u >= a) {
      const float ss = red[u][0][0] + red[u][0][1] + red[u][0][2] + red[u][0][3];
      float o = ov[u] * rsqrtf(ss / (float)p.dv + p.eps);
      o = __bfloat162float(__float2bfloat16(o)) * nw;
      o = o * silu(zz[u]);
      p.out[(long long)(t0 + u - a) * p.Hv * p.dv + h * p.dv + j] = __float2bfloat16(o);
    }
  }
  gdn_mark(tr, 7);
  // ---- pass 2 (tensor cores): S_w = G_w S0 + K C; warp w: state rows 32w .. 32w+31 ----
  if (w >= 0) {
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {  // 32-column blocks
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int i0 = 32 * warp + 16 * mt;
        uint32_t a0, a1, a2, a3;  // A[i][s] = k_s[i] (transposed read of the k rows of sA)
        {
          const int mi = lane >> 3;
          const int srow = (mi >> 1) * 8 + (lane & 7);
          ldsm4t(sA_a + sw16(srow, (i0 + (mi & 1) * 8) >> 3), a0, a1, a2, a3);
        }
        float acc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int col = 32 * cb + 8 * nt + 2 * (lane & 3);
          const int ra = i0 + (lane >> 2), rb = ra + 8;
          const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(sS + sw16(ra, col >> 3) + (col & 7) * 2);
          const __nv_bfloat162 y = *reinterpret_cast<const __nv_bfloat162*>(sS + sw16(rb, col >> 3) + (col & 7) * 2);
          const float2 fx = __bfloat1622float2(x), fy = __bfloat1622float2(y);
          acc[nt][0] = Gw * fx.x;
          acc[nt][1] = Gw * fx.y;
          acc[nt][2] = Gw * fy.x;
          acc[nt][3] = Gw * fy.y;
        }
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          uint32_t b0, b1, b2, b3;
          const int krow = (lane & 7) + ((lane >> 3) & 1) * 8;
          ldsm4t(sC_a + sw16(krow, (32 * cb + 16 * pr) / 8 + (lane >> 4)), b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * pr], a0, a1, a2, a3, b0, b1);
          mma_bf16_16816(acc[2 * pr + 1], a0, a1, a2, a3, b2, b3);
        }
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int col = 32 * cb + 8 * nt + 2 * (lane & 3);
          const int ra = i0 + (lane >> 2), rb = ra + 8;
          *reinterpret_cast<__nv_bfloat162*>(sS + sw16(ra, col >> 3) + (col & 7) * 2) =
              __floats2bfloat162_rn(acc[nt][0], acc[nt][1]);
          *reinterpret_cast<__nv_bfloat162*>(sS + sw16(rb, col >> 3) + (col & 7) * 2) =
              __floats2bfloat162_rn(acc[nt][2], acc[nt][3]);
        }
      }
    }
    __syncthreads();
    gdn_mark(tr, 8);
    uint4* dst = reinterpret_cast<uint4*>(st);
#pragma unroll 4
    for (int v = tid; v < kD * 16; v += kDecThreads) {
      const int row = v >> 4, ch = v & 15;
      dst[v] = *reinterpret_cast<const uint4*>(sS + sw16(row, ch));
    }
  }
  gdn_mark(tr, 9);
}

}  // namespace
}  // namespace oscar

// Install (or, with nullptr, remove) the per-CTA phase timeline of the decode kernel.
extern "C" int oscar_gdn_trace(unsigned long long* buf) {
  return (int)cudaMemcpyToSymbol(oscar::g_gdn_trace, &buf, sizeof(buf));
}

extern "C" int oscar_gdn_step(const oscar::GdnParams* params, int smem_state, cudaStream_t stream) {
  using namespace oscar;
  const GdnParams& p = *params;
  if (p.R <= 0) return 0;
  if (p.dk != kD || p.dv != kD) return -500;
  dim3 grid(p.R, p.Hv);
  if (smem_state) {
    // long prefill chunks: fp32 state in shared memory across 16-token chunks
    const int smem = kD * kD * sizeof(float);
    OSCAR_RC(ensure_smem(gdn_chunk_kernel<16, true>, smem));
    gdn_chunk_kernel<16, true><<<grid, kThreads, smem, stream>>>(p);
  } else if (smem_state == 0 && p.P <= kDecC) {
    // decode / verify: <= 8 tokens per request (commits + new) on the tensor cores
    gdn_decode_kernel<<<grid, kDecThreads, 0, stream>>>(p);
  } else {
    const int smem = kD * kD * sizeof(__nv_bfloat16);
    gdn_chunk_kernel<8, false><<<grid, kThreads, smem, stream>>>(p);
  }
  return (int)cudaGetLastError();
}
