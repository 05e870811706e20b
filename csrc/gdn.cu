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

}  // namespace
}  // namespace oscar

extern "C" int oscar_gdn_step(const oscar::GdnParams* params, int smem_state, cudaStream_t stream) {
  using namespace oscar;
  const GdnParams& p = *params;
  if (p.R <= 0) return 0;
  if (p.dk != kD || p.dv != kD) return -500;
  dim3 grid(p.R, p.Hv);
  if (smem_state) {
    // long prefill chunks: fp32 state in shared memory across 16-token chunks
    static bool attr = false;
    const int smem = kD * kD * sizeof(float);
    if (!attr) {
      OSCAR_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel<16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr = true;
    }
    gdn_chunk_kernel<16, true><<<grid, kThreads, smem, stream>>>(p);
  } else {
    // decode / verify: one chunk of <= 8 tokens per request (commits + new), bf16 staging
    const int smem = kD * kD * sizeof(__nv_bfloat16);
    gdn_chunk_kernel<8, false><<<grid, kThreads, smem, stream>>>(p);
  }
  return (int)cudaGetLastError();
}
