// Paged multi-query GQA attention over BF16 KV pages (the MTP draft layer's shadow
// cache), the dispatch of INT2 pages to the code-domain kernels, and the SIMT
// split-KV merge used when no output rotation is needed.
//
// Work decomposition: one CTA per (work item, KV head).  A work item is
// (request, 64-row block, KV token range); the 64 rows of a block are
// (query token, head-in-group) pairs row = t * g + h, so all g query heads that
// share a KV head read each KV tile once.  Each KV tile of 64 tokens is built in
// shared memory as fp16 by the whole CTA from its source:
//   * position >= prefix                  -> unquantised k/v of the current chunk
//   * otherwise                            -> BF16 page
// which reproduces the reference read semantics (paged_attention.py:136-260).
// Scores and P.V run on the tensor cores (m16n8k16, fp32 accumulate) with an
// online softmax; each CTA writes a normalised partial output and its LSE.
#include "common.cuh"
#include "params.h"
#include "oscar_attention.h"
#include <cstddef>

#include <mutex>

namespace oscar {



namespace {

constexpr int kRows = 64;
constexpr int kTile = 64;
constexpr int kD = 256;
constexpr int kRowBytes = kD * 2;  // fp16 row of a tile
constexpr int kThreads = 128;
constexpr int kPage = 128;
constexpr float kLog2e = 1.4426950408889634f;

OSCAR_DEVICE uint32_t swz(int row, int chunk) {  // byte offset of a 16 B chunk in a 512 B row
  return row * kRowBytes + ((chunk ^ (row & 7)) << 4);
}

OSCAR_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OSCAR_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OSCAR_DEVICE void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
OSCAR_DEVICE uint32_t h2_u32(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct TileCtx {
  int req, hk, prefix, q0, kv_end;
  const int* bt;
};

// Source of one (token, half) owned by a thread.
struct RawInt2 {
  int kind;  // 0 invalid, 2 fresh, 4 bf16
  int blk, off, srow;
};

OSCAR_DEVICE void load_raw(const AttnParams& p, const TileCtx& c, int pos, int half, RawInt2& r) {
  r.kind = 0;
  if (pos >= c.kv_end) return;
  if (pos >= c.prefix) {
    r.kind = 2;
    return;
  }
  const int page = pos / kPage, off = pos % kPage;
  const int blk = c.bt[page];
  r.blk = blk;
  r.off = off;
  r.kind = 4;  // BF16 page (INT2 pages and their staging are read by the code-domain kernels)
}

// Write one thread's (token, half) = 128 dims of K and V into the fp16 tiles.
OSCAR_DEVICE void store_tile(const AttnParams& p, const TileCtx& c, int tok, int pos, int half,
                             const RawInt2& r, uint8_t* ks, uint8_t* vs) {
  const int d0 = half * 128;
  const int chunk0 = d0 / 8;
  if (r.kind == 0) {
    const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<uint4*>(ks + swz(tok, chunk0 + j)) = zero;
      *reinterpret_cast<uint4*>(vs + swz(tok, chunk0 + j)) = zero;
    }
    return;
  }
  if (r.kind == 2) {
    const long long t = c.q0 + (pos - c.prefix);
    const uint4* kf = reinterpret_cast<const uint4*>(p.k_fresh + (t * p.Hk + c.hk) * p.D + d0);
    const uint4* vf = reinterpret_cast<const uint4*>(p.v_fresh + (t * p.Hk + c.hk) * p.D + d0);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<uint4*>(ks + swz(tok, chunk0 + j)) = __ldg(kf + j);
      *reinterpret_cast<uint4*>(vs + swz(tok, chunk0 + j)) = __ldg(vf + j);
    }
    return;
  }
  // kind 4: BF16 page
  const long long base = ((long long)(r.blk * kPage + r.off) * p.Hk + c.hk) * p.D + d0;
  const uint4* kb = reinterpret_cast<const uint4*>(p.kc + base);
  const uint4* vb = reinterpret_cast<const uint4*>(p.vc + base);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint4 a = __ldg(kb + j), b = __ldg(vb + j);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
    uint4 ka, va;
    uint32_t* pka = reinterpret_cast<uint32_t*>(&ka);
    uint32_t* pva = reinterpret_cast<uint32_t*>(&va);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(pa[e]);
      const float2 fb = __bfloat1622float2(pb[e]);
      pka[e] = h2_u32(fa.x, fa.y);
      pva[e] = h2_u32(fb.x, fb.y);
    }
    *reinterpret_cast<uint4*>(ks + swz(tok, chunk0 + j)) = ka;
    *reinterpret_cast<uint4*>(vs + swz(tok, chunk0 + j)) = va;
  }
}

__global__ void __launch_bounds__(kThreads, 2) paged_attention_kernel(AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* qs = smem;                       // [64][256] fp16
  uint8_t* ks = smem + kRows * kRowBytes;   // [64][256]
  uint8_t* vs = ks + kTile * kRowBytes;     // [64][256]
  const int item = blockIdx.x, hk = blockIdx.y;
  const int4 w = p.work[item];
  const int req = w.x, row0 = w.y, kv_begin = w.z, kv_end_item = w.w;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.Hq / p.Hk;
  const int q0 = p.q_start[req];
  const int qlen = p.q_start[req + 1] - q0;
  const int seq = p.seq_lens[req];
  TileCtx c;
  c.req = req;
  c.hk = hk;
  c.prefix = seq - qlen;
  c.q0 = q0;
  c.kv_end = kv_end_item;
  c.bt = p.block_tables + (long long)req * p.bt_stride;

  // ---- Q tile -----------------------------------------------------------------------
  for (int idx = tid; idx < kRows * 32; idx += kThreads) {
    const int r = idx >> 5, ch = idx & 31;
    const int gr = row0 + r;
    const int t = gr / g, h = gr % g;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < qlen) v = __ldg(reinterpret_cast<const uint4*>(p.q + ((long long)(q0 + t) * p.Hq + hk * g + h) * kD) + ch);
    *reinterpret_cast<uint4*>(qs + swz(r, ch)) = v;
  }

  // Per-thread row bookkeeping: rows ra = warp*16 + lane/4 and rb = ra + 8.
  const int ra = warp * 16 + (lane >> 2), rb = ra + 8;
  const int ta = (row0 + ra) / g, tb = (row0 + rb) / g;
  const int lim_a = ta < qlen ? c.prefix + ta : -1;  // last visible key position
  const int lim_b = tb < qlen ? c.prefix + tb : -1;
  const float sl2 = p.scale * kLog2e;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[32][4];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  const uint32_t qs_a = smem_u32(qs), ks_a = smem_u32(ks), vs_a = smem_u32(vs);

  // Highest key position any row of this block may see.
  int row_last = min(row0 + kRows, qlen * g) - 1;
  const int kv_stop = min(kv_end_item, row_last >= 0 ? c.prefix + row_last / g + 1 : 0);
  c.kv_end = kv_stop;
  const int ntiles = kv_stop > kv_begin ? (kv_stop - kv_begin + kTile - 1) / kTile : 0;

  const int my_tok = tid >> 1, my_half = tid & 1;
  RawInt2 raw;
  if (ntiles > 0) load_raw(p, c, kv_begin + my_tok, my_half, raw);

  for (int it = 0; it < ntiles; ++it) {
    const int tile0 = kv_begin + it * kTile;
    __syncthreads();  // previous tile fully consumed
    store_tile(p, c, my_tok, tile0 + my_tok, my_half, raw, ks, vs);
    __syncthreads();
    if (it + 1 < ntiles) load_raw(p, c, tile0 + kTile + my_tok, my_half, raw);

    // ---- S = Q K^T for this warp's 16 rows x 64 tokens ----
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = 2 * kk + (lane >> 4);
        ldsm_x4(qs_a + swz(r, ch), a0, a1, a2, a3);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int tr = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int ch = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(ks_a + swz(tr, ch), b0, b1, b2, b3);
        mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- online softmax ----
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int pos = tile0 + j * 8 + 2 * (lane & 3);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int pp = pos + e;
        const bool va = pp <= lim_a && pp < kv_stop;
        const bool vb = pp <= lim_b && pp < kv_stop;
        s[j][e] = va ? s[j][e] * sl2 : -INFINITY;
        s[j][2 + e] = vb ? s[j][2 + e] * sl2 : -INFINITY;
        mx_a = fmaxf(mx_a, s[j][e]);
        mx_b = fmaxf(mx_b, s[j][2 + e]);
      }
    }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, o2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, o2));
    }
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float base_a = mn_a == -INFINITY ? 0.f : mn_a;
    const float base_b = mn_b == -INFINITY ? 0.f : mn_b;
    const float ca = exp2f(m_a - base_a), cb = exp2f(m_b - base_b);
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(s[j][0] - base_a);
      s[j][1] = exp2f(s[j][1] - base_a);
      s[j][2] = exp2f(s[j][2] - base_b);
      s[j][3] = exp2f(s[j][3] - base_b);
      sum_a += s[j][0] + s[j][1];
      sum_b += s[j][2] + s[j][3];
    }
    l_a = l_a * ca + sum_a;
    l_b = l_b * cb + sum_b;
    m_a = mn_a;
    m_b = mn_b;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      o[j][0] *= ca;
      o[j][1] *= ca;
      o[j][2] *= cb;
      o[j][3] *= cb;
    }
    // ---- O += P V ----
#pragma unroll
    for (int sg = 0; sg < 4; ++sg) {
      const uint32_t a0 = h2_u32(s[2 * sg][0], s[2 * sg][1]);
      const uint32_t a1 = h2_u32(s[2 * sg][2], s[2 * sg][3]);
      const uint32_t a2 = h2_u32(s[2 * sg + 1][0], s[2 * sg + 1][1]);
      const uint32_t a3 = h2_u32(s[2 * sg + 1][2], s[2 * sg + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int tr = sg * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = 2 * dp + (lane >> 4);
        ldsm_x4_t(vs_a + swz(tr, ch), b0, b1, b2, b3);
        mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }

  // ---- finalise: row sums across the 4 lanes of a row, normalise, write partials ----
#pragma unroll
  for (int o2 = 1; o2 <= 2; o2 <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o2);
  }
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  float* po = p.part_o + ((long long)item * p.Hk + hk) * kRows * kD;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int d = j * 8 + 2 * (lane & 3);
    *reinterpret_cast<float2*>(po + ra * kD + d) = make_float2(o[j][0] * inv_a, o[j][1] * inv_a);
    *reinterpret_cast<float2*>(po + rb * kD + d) = make_float2(o[j][2] * inv_b, o[j][3] * inv_b);
  }
  if ((lane & 3) == 0) {
    float* pl = p.part_lse + ((long long)item * p.Hk + hk) * kRows;
    pl[ra] = l_a > 0.f ? (m_a + log2f(l_a)) / kLog2e : -INFINITY;
    pl[rb] = l_b > 0.f ? (m_b + log2f(l_b)) / kLog2e : -INFINITY;
  }
}

// ------------------------------------------------------------------ merge
// One CTA (256 threads, thread = output dim) per query token.
__global__ void __launch_bounds__(256) attn_merge_kernel(MergeParams p) {
  extern __shared__ float msm[];
  float* orot = msm;  // [Hq][D]
  __shared__ float red[8];
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  const int D = p.D, Hq = p.Hq, g = p.Hq / p.Hk;
  const int req = p.tok_req[t];
  const int tt = t - p.q_start[req];
  // combine the split partials of every head
  for (int h = 0; h < Hq; ++h) {
    const int hk = h / g, hg = h % g;
    const int row = tt * g + hg;
    const int rb = row / kRows, r = row % kRows;
    const int first = p.item_first[req * p.max_rb + rb];
    const int cnt = p.item_count[req * p.max_rb + rb];
    float mx = -INFINITY;
    for (int s = 0; s < cnt; ++s) mx = fmaxf(mx, p.part_lse[((long long)(first + s) * p.Hk + hk) * kRows + r]);
    float acc = 0.f, wsum = 0.f;
    if (mx > -INFINITY) {
      for (int s = 0; s < cnt; ++s) {
        const long long base = ((long long)(first + s) * p.Hk + hk) * kRows + r;
        const float wgt = __expf(p.part_lse[base] - mx);
        wsum += wgt;
        if (tid < D) acc = fmaf(wgt, p.part_o[base * kD + tid], acc);
      }
    }
    if (tid < D) orot[h * D + tid] = wsum > 0.f ? acc / wsum : 0.f;
  }
  __syncthreads();
  // rotate back (o = o_rot @ R_v^T), gate, and collect the token's absmax
  float amax = 0.f;
  constexpr int kHB = 8;
  for (int h0 = 0; h0 < Hq; h0 += kHB) {
    float acc[kHB];
#pragma unroll
    for (int j = 0; j < kHB; ++j) acc[j] = 0.f;
    const int nh = min(kHB, Hq - h0);
    if (tid < D) {
      if (p.RvT) {
        for (int i = 0; i < D; ++i) {
          const float rv = __ldg(p.RvT + (long long)i * D + tid);
#pragma unroll
          for (int j = 0; j < kHB; ++j)
            if (j < nh) acc[j] = fmaf(orot[(h0 + j) * D + i], rv, acc[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < kHB; ++j)
          if (j < nh) acc[j] = orot[(h0 + j) * D + tid];
      }
#pragma unroll
      for (int j = 0; j < kHB; ++j) {
        if (j >= nh) break;
        float v = acc[j];
        if (p.gate) v *= sigmoidf_(__bfloat162float(p.gate[(long long)t * p.gate_ld + (h0 + j) * p.gate_hstride + tid]));
        // round like a bf16 activation before quantisation
        v = __bfloat162float(__float2bfloat16(v));
        acc[j] = v;
        amax = fmaxf(amax, fabsf(v));
        if (p.out_bf16) p.out_bf16[(long long)t * Hq * D + (h0 + j) * D + tid] = __float2bfloat16(v);
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kHB; ++j)
      if (j < nh && tid < D) orot[(h0 + j) * D + tid] = acc[j];
    __syncthreads();
  }
  if (p.out_i8) {
    amax = block_max<8>(amax, red);
    const float sc = amax > 0.f ? amax / 127.f : 1.f;
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    if (tid < D)
      for (int h = 0; h < Hq; ++h) p.out_i8[(long long)t * Hq * D + h * D + tid] = quant_i8(orot[h * D + tid], inv);
    if (tid == 0) p.out_scale[t] = sc;
  }
}

}  // namespace
}  // namespace oscar

extern "C" int oscar_int2_attention(const oscar::AttnParams* params, cudaStream_t stream);

extern "C" int oscar_params_layout(long long* out, int cap) {
  using oscar::AttnParams;
  using oscar::MergeParams;
#define OSCAR_A(f) (long long)offsetof(AttnParams, f)
#define OSCAR_M(f) (long long)offsetof(MergeParams, f)
  const long long v[] = {
      (long long)sizeof(AttnParams), OSCAR_A(q), OSCAR_A(k_fresh), OSCAR_A(v_fresh), OSCAR_A(Hq), OSCAR_A(Hk),
      OSCAR_A(D), OSCAR_A(scale), OSCAR_A(kv_mode), OSCAR_A(pool), OSCAR_A(page_bytes), OSCAR_A(kc), OSCAR_A(vc),
      OSCAR_A(stage_k), OSCAR_A(stage_v), OSCAR_A(owner), OSCAR_A(stage_rows), OSCAR_A(block_tables),
      OSCAR_A(bt_stride), OSCAR_A(q_start), OSCAR_A(seq_lens), OSCAR_A(work), OSCAR_A(n_work), OSCAR_A(part_o),
      OSCAR_A(part_lse), OSCAR_A(status), OSCAR_A(stage_req_slot), OSCAR_A(stage_sink), OSCAR_A(stage_ring),
      (long long)sizeof(MergeParams), OSCAR_M(part_o), OSCAR_M(part_lse), OSCAR_M(item_first), OSCAR_M(item_count),
      OSCAR_M(max_rb), OSCAR_M(tok_req), OSCAR_M(q_start), OSCAR_M(Hq), OSCAR_M(Hk), OSCAR_M(D), OSCAR_M(RvT),
      OSCAR_M(gate), OSCAR_M(gate_ld), OSCAR_M(gate_hstride), OSCAR_M(out_bf16), OSCAR_M(out_i8),
      OSCAR_M(out_scale), OSCAR_M(T)};
#undef OSCAR_A
#undef OSCAR_M
  const int n = (int)(sizeof(v) / sizeof(v[0]));
  for (int i = 0; i < n && i < cap; ++i) out[i] = v[i];
  return n;
}

extern "C" int oscar_paged_attention(const oscar::AttnParams* params, cudaStream_t stream) {
  using namespace oscar;
  const AttnParams& p = *params;
  if (p.n_work <= 0) return 0;
  if (p.kv_mode == 0) return oscar_int2_attention(params, stream);  // pipelined code-domain kernel
  if (p.D != kD) return -300;
  const size_t smem = (kRows + 2 * kTile) * kRowBytes;
  OSCAR_RC(ensure_smem(paged_attention_kernel, (int)smem));
  dim3 grid(p.n_work, p.Hk);
  paged_attention_kernel<<<grid, kThreads, smem, stream>>>(p);
  return (int)cudaGetLastError();
}

extern "C" int oscar_attn_merge(const oscar::MergeParams* params, cudaStream_t stream) {
  using namespace oscar;
  const MergeParams& p = *params;
  if (p.T <= 0) return 0;
  if (p.D != kD) return -301;
  const size_t smem = (size_t)p.Hq * p.D * sizeof(float);
  OSCAR_RC(ensure_smem(attn_merge_kernel, 200 * 1024));
  attn_merge_kernel<<<p.T, 256, smem, stream>>>(p);
  return (int)cudaGetLastError();
}

// ============================================================================
// No-allocation entry point.
//
// This entry point has no counterpart in the reference (which has no CUDA code).
// It serves callers that cannot allocate device memory at the time they launch
// attention: code running inside a custom allocator or memory-pool callback,
// embedders whose runtime forbids cudaMalloc on the serving path (it can
// synchronise the device and stall other streams), and hosts that must run with
// a fixed memory footprint decided at start-up.  Such callers pass their inputs
// and outputs exactly as for oscar_paged_attention + oscar_attn_merge, but no
// workspace: the split-KV partial results live in a fixed device array that is
// part of this library's image.
//
// Limits and contract:
//   * the scratch holds at most kNoAllocItems (work item x KV head) partials of
//     64 rows x 256 dims in fp32 (16 MiB) plus their log-sum-exps (64 KiB); a call
//     with n_work * Hk above that is rejected with -310 before anything launches;
//   * every GPU that loads this library keeps those 16.06 MiB until the process
//     exits;
//   * every call on a device shares the same array and leaves its contents
//     behind; each call overwrites every partial it later reads, so nothing needs
//     to start at zero, but calls whose kernels overlap on the GPU (different
//     streams without ordering between them) race on the array and must be
//     serialised by the caller;
//   * the first call on each device resolves the array's device address with
//     cudaGetSymbolAddress while that device is current; make that first call
//     before any stream capture;
//   * the entry point itself calls no cudaMalloc, cudaFree or other allocating
//     routine.
// ============================================================================
namespace oscar {
namespace {
constexpr int kNoAllocItems = OSCAR_NOALLOC_MAX_ITEMS;
constexpr size_t kNoAllocPartO = (size_t)kNoAllocItems * kRows * kD;  // floats
constexpr size_t kNoAllocPartL = (size_t)kNoAllocItems * kRows;       // floats
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocPartO + kNoAllocPartL];

constexpr int kMaxDevices = 64;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return -311;
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}
}  // namespace
}  // namespace oscar

// Same inputs and outputs as oscar_paged_attention followed by oscar_attn_merge;
// the part_o / part_lse fields of both parameter blocks are ignored.
extern "C" int oscar_paged_attention_noalloc(const oscar::AttnParams* attn, const oscar::MergeParams* merge,
                                             cudaStream_t stream) {
  using namespace oscar;
  if (!attn || !merge) return -312;
  if (attn->n_work <= 0 || merge->T <= 0) return 0;
  if (attn->D != kD || merge->D != kD) return -300;
  if ((long long)attn->n_work * attn->Hk > kNoAllocItems) return -310;
  float* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  AttnParams a = *attn;
  a.part_o = scratch;
  a.part_lse = scratch + kNoAllocPartO;
  MergeParams m = *merge;
  m.part_o = a.part_o;
  m.part_lse = a.part_lse;
  rc = oscar_paged_attention(&a, stream);
  if (rc) return rc;
  return oscar_attn_merge(&m, stream);
}
