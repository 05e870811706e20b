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
// per (request, value head); thread j owns column j.
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
constexpr int kC = 16;   // tokens per chunk
constexpr int kThreads = 128;

OSCAR_DEVICE float softplusf(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

template <bool kSmemState>
__global__ void __launch_bounds__(kThreads) gdn_chunk_kernel(GdnParams p) {
  extern __shared__ float sS[];  // [dk][dv] fp32 when kSmemState
  __shared__ float qc[kC][kD], kc[kC][kD];
  __shared__ float KK[kC][kC], KQ[kC][kC];
  __shared__ float Lg[kC], Bt[kC];
  __shared__ float nrm[kC][2], red[kC][4];
  __shared__ float pb_b[kC], pb_a[kC];

  const int req = blockIdx.x, h = blockIdx.y;
  const int j = threadIdx.x, lane = j & 31, warp = j >> 5;
  const int t0 = p.q_start[req], T = p.q_start[req + 1] - t0;
  const int a = p.n_commit[req];
  const int n_all = a + T;
  if (n_all <= 0) return;
  const bool keep = p.keep_pending[req] != 0;
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

  if (a > p.P || a > kC || (keep && (n_all > kC || T > p.P))) {
    if (j == 0) record_status(p.status, kBadShape);
    return;
  }
  // gate inputs of the tokens to commit, read before this CTA overwrites them
  if (j < a) {
    pb_b[j] = __bfloat162float(pb[j * 2 * p.Hv + h]);
    pb_a[j] = __bfloat162float(pb[j * 2 * p.Hv + p.Hv + h]);
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

  if (kSmemState) {
    for (int i = 0; i < kD; ++i) sS[i * kD + j] = __bfloat162float(st[i * p.dv + j]);
  }
  __syncthreads();

  bool conv_saved = false;
  auto save_conv = [&]() {
    if (hh == 0)
      for (int i = 0; i < 3; ++i) {
        cs_out[cq * 3 + i] = __float2bfloat16(wq[i]);
        cs_out[ck * 3 + i] = __float2bfloat16(wk[i]);
      }
    for (int i = 0; i < 3; ++i) cs_out[cv * 3 + i] = __float2bfloat16(wv[i]);
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
      if (u >= n) continue;
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
        if (keep) {
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
      qc[u][j] = silu(q);
      kc[u][j] = silu(k);
      vv[u] = silu(v);
      if (j == 0) {
        Bt[u] = sigmoidf_(braw);
        Lg[u] = A * softplusf(araw + dtb);  // log g
      }
    }
    __syncthreads();
    // ---- L2 norms of q and k per token (warp w: tokens w, w+4, ...) ----
    for (int u = warp; u < n; u += 4) {
      float sq = 0.f, sk = 0.f;
      for (int i = lane; i < kD; i += 32) {
        sq += qc[u][i] * qc[u][i];
        sk += kc[u][i] * kc[u][i];
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      if (lane == 0) {
        nrm[u][0] = rsqrtf(sq + 1e-6f) * qscale;
        nrm[u][1] = rsqrtf(sk + 1e-6f);
      }
    }
    if (j == 0)
      for (int u = 1; u < n; ++u) Lg[u] += Lg[u - 1];  // cumulative log decay
    __syncthreads();
    for (int u = 0; u < n; ++u) {
      qc[u][j] *= nrm[u][0];
      kc[u][j] *= nrm[u][1];
    }
    for (int u = n; u < kC; ++u) {
      qc[u][j] = 0.f;
      kc[u][j] = 0.f;
    }
    __syncthreads();
    // ---- pairwise dot products k_s.k_t and k_s.q_t for s <= t ----
    for (int pr = warp; pr < n * n; pr += 4) {
      const int s_ = pr / n, t_ = pr % n;
      if (s_ > t_) continue;
      float kk = 0.f, kq = 0.f;
      for (int i = lane; i < kD; i += 32) {
        kk += kc[s_][i] * kc[t_][i];
        kq += kc[s_][i] * qc[t_][i];
      }
      kk = warp_sum(kk);
      kq = warp_sum(kq);
      if (lane == 0) {
        KK[s_][t_] = kk;
        KQ[s_][t_] = kq;
      }
    }
    __syncthreads();
    // ---- pass 1: S0^T k_t and S0^T q_t for column j ----
    float kvS[kC], qS[kC];
#pragma unroll
    for (int u = 0; u < kC; ++u) kvS[u] = qS[u] = 0.f;
    for (int i = 0; i < kD; ++i) {
      const float sv = kSmemState ? sS[i * kD + j] : __bfloat162float(st[i * p.dv + j]);
#pragma unroll
      for (int u = 0; u < kC; ++u) {
        kvS[u] = fmaf(sv, kc[u][i], kvS[u]);
        qS[u] = fmaf(sv, qc[u][i], qS[u]);
      }
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
      const float ss = warp_sum(o * o);
      if (lane == 0) red[u][warp] = ss;
    }
    __syncthreads();
    // ---- gated RMSNorm over dv and output ----
#pragma unroll
    for (int u = 0; u < kC; ++u) {
      if (u < n && c0 + u >= a) {
        const float ss = red[u][0] + red[u][1] + red[u][2] + red[u][3];
        float o = ov[u] * rsqrtf(ss / (float)p.dv + p.eps);
        o = __bfloat162float(__float2bfloat16(o)) * nw;
        o = o * silu(zz[u]);
        p.out[(long long)(t0 + c0 + u - a) * p.Hv * p.dv + h * p.dv + j] = __float2bfloat16(o);
      }
    }
    // ---- pass 2: state after token w of this chunk ----
    const int w = min(n - 1, write_after - c0);
    if (w >= 0) {
      const float Gw = __expf(Lg[w]);
      float cf[kC];
#pragma unroll
      for (int s_ = 0; s_ < kC; ++s_) cf[s_] = (s_ <= w) ? __expf(Lg[w] - Lg[s_]) * dd[s_] : 0.f;
      for (int i = 0; i < kD; ++i) {
        float v = Gw * (kSmemState ? sS[i * kD + j] : __bfloat162float(st[i * p.dv + j]));
#pragma unroll
        for (int s_ = 0; s_ < kC; ++s_) v = fmaf(kc[s_][i], cf[s_], v);
        if (kSmemState) sS[i * kD + j] = v;
        else st[i * p.dv + j] = __float2bfloat16(v);
      }
    }
    __syncthreads();
    if (write_after < c0 + n) break;  // the stored state ends inside this chunk
  }
  if (kSmemState) {
    for (int i = 0; i < kD; ++i) st[i * p.dv + j] = __float2bfloat16(sS[i * kD + j]);
  }
  if (!conv_saved) save_conv();
}

}  // namespace
}  // namespace oscar

extern "C" int oscar_gdn_step(const oscar::GdnParams* params, int smem_state, cudaStream_t stream) {
  using namespace oscar;
  const GdnParams& p = *params;
  if (p.R <= 0) return 0;
  if (p.dk != kD || p.dv != kD) return -500;
  dim3 grid(p.R, p.Hv);
  if (smem_state) {
    static bool attr = false;
    const int smem = kD * kD * sizeof(float);
    if (!attr) {
      OSCAR_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr = true;
    }
    gdn_chunk_kernel<true><<<grid, kThreads, smem, stream>>>(p);
  } else {
    gdn_chunk_kernel<false><<<grid, kThreads, 0, stream>>>(p);
  }
  return (int)cudaGetLastError();
}
