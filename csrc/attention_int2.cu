// INT2 paged multi-query attention, pipelined (v2).
//
// One CTA per (work item, KV head); the work item is (request, <= 64 query rows,
// page-aligned KV range).  Eight warps: each owns one 16-row tile of the queries
// and a slice of every 64-token KV tile (16 tokens with <= 2 row tiles, 32 with 4)
// and keeps its own online-softmax state; the states are merged in shared memory
// at the end, so every warp issues tensor-core work on every tile.  Thread 0 streams whole page-heads (17,408 B of codes and
// fp16 scale/zero) plus the page's 128 staging owner tags into a 4-deep shared-memory
// ring with bulk asynchronous copies (plain CTA-local copies; no cluster multicast),
// so up to three pages are in flight while the CTA computes on the fourth.
//
// Scores and P.V run directly on the 2-bit codes.  With per-token asymmetric
// scale s and zero z,
//     q . k_j = s_j (q . c_j) + z_j sum(q)        sum_j p_j v_j = sum_j (p_j s_j) c_j + sum_j p_j z_j
// so K and V tiles hold the exact codes c (widened to fp16 with one logic op per
// pair, see mma::codes_to_h2), the tensor cores compute q.c and (p*s).c, and the
// scale/zero terms are applied per column on the score and probability fragments.
// Tokens that are not INT2 - the current chunk (unquantised k/v) and staged
// sink/recent tokens (fp32, owner tag == physical block) - are written into the
// same tiles as fp16 values with s = 1, z = 0, which reproduces the reference read
// semantics (paged_attention.py:136-260) without a second pass.
#include "common.cuh"
#include "mma.cuh"
#include "params.h"
#include "sm100.cuh"

namespace oscar {
namespace {

constexpr int kRows = 64;
constexpr int kTile = 64;
constexpr int kD = 256;
constexpr int kPage = 128;
constexpr int kThreads = 256;  // 8 warps: row tiles x token groups
constexpr int kRing = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitNs = 2000000000ull;

struct Smem {
  int ring_off, slot_bytes, ktile, vtile, qtile, tokp, sq, bars, misc, total;
};

__host__ __device__ inline Smem smem_layout(int page_bytes) {
  Smem s;
  s.slot_bytes = ((page_bytes + 15) / 16) * 16 + kPage * 4;  // page + owner tags
  s.ring_off = 0;
  s.ktile = kRing * s.slot_bytes;
  s.vtile = s.ktile + kTile * mma::kRowBytes;
  s.qtile = s.vtile + kTile * mma::kRowBytes;
  s.tokp = s.qtile + kRows * mma::kRowBytes;  // float4 (ks, kz, vs, vz) per tile token
  s.sq = s.tokp + kTile * 16;                 // sum(q) per row
  s.bars = s.sq + kRows * 4;                  // kRing mbarriers
  s.misc = s.bars + kRing * 8;                // block id per ring slot
  s.total = s.misc + kRing * 4 + 16;
  return s;
}

// V^T tile: 256 dim rows of 64 tokens (128 B), 16 B chunks XOR-swizzled by row.
OSCAR_DEVICE uint32_t swz_vt(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// One warp's share of a 64-token tile: S = Q C^T for its 16 rows and TOK tokens,
// online softmax, O += P' C_v.  Columns of the tile are tokens tok0 .. tok0+TOK-1.
template <int TOK>
OSCAR_DEVICE void warp_tile(const uint32_t qs_a, const uint32_t ks_a, const uint32_t vs_a, const float4* tokp,
                            int row_base, int tok0, int tile0, int kv_begin, int kv_stop, int lim_a, int lim_b,
                            float sq_a, float sq_b, float sl2, float& m_a, float& m_b, float& l_a, float& l_b,
                            float& z_a, float& z_b, float (&o)[32][4]) {
  constexpr int NT = TOK / 8;   // n8 tiles of scores
  constexpr int KS = TOK / 16;  // k16 slices of P.V
  const int lane = threadIdx.x & 31;
  float sacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 16; ++kk) {
    uint32_t a0, a1, a2, a3;
    mma::ldsm_x4(qs_a + mma::swz(row_base + (lane & 7) + ((lane >> 3) & 1) * 8, 2 * kk + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
    for (int np = 0; np < KS; ++np) {
      uint32_t b0, b1, b2, b3;
      mma::ldsm_x4(ks_a + mma::swz(tok0 + np * 16 + (lane & 7) + (lane >> 4) * 8, 2 * kk + ((lane >> 3) & 1)), b0, b1,
                   b2, b3);
      mma::mma_f16(sacc[2 * np], a0, a1, a2, a3, b0, b1);
      mma::mma_f16(sacc[2 * np + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  float mx_a = -INFINITY, mx_b = -INFINITY;
  float pv[NT][2][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = tok0 + j * 8 + 2 * (lane & 3) + e;
      const int pos = tile0 + col;
      const float4 tp = tokp[col];
      pv[j][e][0] = tp.z;
      pv[j][e][1] = tp.w;
      const bool in = pos >= kv_begin && pos < kv_stop;
      const float sa = fmaf(tp.x, sacc[j][e], tp.y * sq_a) * sl2;
      const float sb = fmaf(tp.x, sacc[j][2 + e], tp.y * sq_b) * sl2;
      sacc[j][e] = (in && pos <= lim_a) ? sa : -INFINITY;
      sacc[j][2 + e] = (in && pos <= lim_b) ? sb : -INFINITY;
      mx_a = fmaxf(mx_a, sacc[j][e]);
      mx_b = fmaxf(mx_b, sacc[j][2 + e]);
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
  const float ca = exp2f(m_a - base_a), cbv = exp2f(m_b - base_b);
  float sum_a = 0.f, sum_b = 0.f, zs_a = 0.f, zs_b = 0.f;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float pa = exp2f(sacc[j][e] - base_a);
      const float pb = exp2f(sacc[j][2 + e] - base_b);
      sum_a += pa;
      sum_b += pb;
      zs_a = fmaf(pa, pv[j][e][1], zs_a);
      zs_b = fmaf(pb, pv[j][e][1], zs_b);
      sacc[j][e] = pa * pv[j][e][0];  // P' = P * s_v
      sacc[j][2 + e] = pb * pv[j][e][0];
    }
  }
  l_a = l_a * ca + sum_a;
  l_b = l_b * cbv + sum_b;
  z_a = z_a * ca + zs_a;
  z_b = z_b * cbv + zs_b;
  m_a = mn_a;
  m_b = mn_b;
  // rescale the accumulator only when some row's running max moved
  if (__any_sync(0xffffffffu, ca != 1.f || cbv != 1.f)) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      o[j][0] *= ca;
      o[j][1] *= ca;
      o[j][2] *= cbv;
      o[j][3] *= cbv;
    }
  }
#pragma unroll
  for (int sg = 0; sg < KS; ++sg) {
    const uint32_t a0 = mma::h2_u32(sacc[2 * sg][0], sacc[2 * sg][1]);
    const uint32_t a1 = mma::h2_u32(sacc[2 * sg][2], sacc[2 * sg][3]);
    const uint32_t a2 = mma::h2_u32(sacc[2 * sg + 1][0], sacc[2 * sg + 1][1]);
    const uint32_t a3 = mma::h2_u32(sacc[2 * sg + 1][2], sacc[2 * sg + 1][3]);
#pragma unroll
    for (int dp = 0; dp < 16; ++dp) {
      uint32_t b0, b1, b2, b3;
      mma::ldsm_x4(vs_a + swz_vt(dp * 16 + (lane & 7) + (lane >> 4) * 8, ((tok0 + sg * 16) >> 3) + ((lane >> 3) & 1)),
                   b0, b1, b2, b3);
      mma::mma_f16(o[2 * dp], a0, a1, a2, a3, b0, b1);
      mma::mma_f16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) int2_attention_kernel(AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Smem L = smem_layout(p.page_bytes);
  uint8_t* ring = smem + L.ring_off;
  uint8_t* ks = smem + L.ktile;
  uint8_t* vs = smem + L.vtile;
  uint8_t* qs = smem + L.qtile;
  float4* tokp = reinterpret_cast<float4*>(smem + L.tokp);
  float* sqs = reinterpret_cast<float*>(smem + L.sq);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  int* slot_blk = reinterpret_cast<int*>(smem + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc + kRing * 4);

  const int item = blockIdx.x, hk = blockIdx.y;
  const int4 w = p.work[item];
  const int req = w.x, row0 = w.y, kv_begin = w.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.Hq / p.Hk;
  const int q0 = p.q_start[req];
  const int qlen = p.q_start[req + 1] - q0;
  const int seq = p.seq_lens[req];
  const int prefix = seq - qlen;
  const int* bt = p.block_tables + (long long)req * p.bt_stride;
  const int nrows = min(kRows, qlen * g - row0);
  const int kv_stop = min(w.w, nrows > 0 ? prefix + (row0 + nrows - 1) / g + 1 : 0);
  const bool staging = p.stage_rows > 0;
  const uint32_t page_tx = (uint32_t)p.page_bytes + (staging ? kPage * 4 : 0);
  // warp roles: row tile rt, token group tg of every 64-token tile
  const int n_rt = (nrows + 15) / 16;
  const bool four_rt = n_rt > 2;
  const int rt = four_rt ? (warp & 3) : (warp & 1);
  const int tg = four_rt ? (warp >> 2) : (warp >> 1);
  const int tok0 = four_rt ? tg * 32 : tg * 16;
  const bool mma_warp = rt < n_rt;

  if (tid == 0) {
    for (int s = 0; s < kRing; ++s) sm100::mbar_init(&full[s], 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();

  const int p_first = kv_begin / kPage;
  const int n_pages = kv_stop > kv_begin ? (kv_stop - 1) / kPage - p_first + 1 : 0;
  auto issue = [&](int i) {  // page index i of this CTA -> ring slot i % kRing
    const int s = i % kRing;
    const int blk = bt[p_first + i];
    slot_blk[s] = blk;
    uint8_t* dst = ring + s * L.slot_bytes;
    sm100::mbar_arrive_expect_tx(&full[s], page_tx);
    sm100::bulk_load(dst, p.pool + ((long long)blk * p.Hk + hk) * p.page_bytes, p.page_bytes, &full[s]);
    if (staging)
      sm100::bulk_load(dst + ((p.page_bytes + 15) / 16) * 16, p.owner + (long long)stage_row_of(p, req, p_first + i, blk) * kPage,
                       kPage * 4, &full[s]);
  };
  if (tid == 0)
    for (int i = 0; i < min(kRing, n_pages); ++i) issue(i);

  // ---- Q tile (fp16) and per-row sum(q) ----
  for (int idx = tid; idx < kRows * 32; idx += kThreads) {
    const int r = idx >> 5, ch = idx & 31;
    const int gr = row0 + r;
    const int t = gr / g, h = gr % g;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows) v = __ldg(reinterpret_cast<const uint4*>(p.q + ((long long)(q0 + t) * p.Hq + hk * g + h) * kD) + ch);
    *reinterpret_cast<uint4*>(qs + mma::swz(r, ch)) = v;
  }
  __syncthreads();
  if (tid < kRows) {
    float acc = 0.f;
    for (int ch = 0; ch < 32; ++ch) {
      const uint4 v = *reinterpret_cast<const uint4*>(qs + mma::swz(tid, ch));
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        acc += f.x + f.y;
      }
    }
    sqs[tid] = acc;
  }

  const int ra = rt * 16 + (lane >> 2), rb = ra + 8;
  const int ta = (row0 + ra) / g, tb = (row0 + rb) / g;
  const int lim_a = ra < nrows ? prefix + ta : -1;  // last visible key position
  const int lim_b = rb < nrows ? prefix + tb : -1;
  const float sl2 = p.scale * kLog2e;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f, z_a = 0.f, z_b = 0.f;
  float o[32][4];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  const uint32_t qs_a = smem_u32(qs), ks_a = smem_u32(ks), vs_a = smem_u32(vs);
  __syncthreads();
  const float sq_a = sqs[min(ra, kRows - 1)], sq_b = sqs[min(rb, kRows - 1)];

  const int my_tok = tid >> 2, my_q = tid & 3;  // token of the tile, quarter of the dims
  bool ok = true;
  for (int i = 0; i < n_pages && ok; ++i) {
    const int s = i % kRing;
    if (!sm100::mbar_wait(&full[s], (i / kRing) & 1, abort_flag, p.status, kTimeoutTmaFull, kWaitNs)) {
      ok = false;
      break;
    }
    const uint8_t* pg = ring + s * L.slot_bytes;
    const int* own = reinterpret_cast<const int*>(pg + ((p.page_bytes + 15) / 16) * 16);
    const int blk = slot_blk[s];
    const int page_pos = (p_first + i) * kPage;
    for (int half = 0; half < 2; ++half) {
      const int tile0 = page_pos + half * kTile;
      if (tile0 >= kv_stop) break;
      // ---------------- build the code / value tiles (thread: one token, 64 dims) ----------------
      {
        const int j = half * kTile + my_tok;  // token within the page
        const int pos = page_pos + j;
        const int d0 = my_q * 64;
        const int c0 = d0 / 8;
        float4 par = make_float4(0.f, 0.f, 0.f, 0.f);
        bool value_tok = false;
        if (pos >= kv_stop || pos < kv_begin) {
          const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(ks + mma::swz(my_tok, c0 + c)) = z;
        } else if (pos >= prefix) {  // current chunk: unquantised fp16
          const long long t = q0 + (pos - prefix);
          const uint4* kf = reinterpret_cast<const uint4*>(p.k_fresh + (t * p.Hk + hk) * kD + d0);
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(ks + mma::swz(my_tok, c0 + c)) = __ldg(kf + c);
          par = make_float4(1.f, 0.f, 1.f, 0.f);
          value_tok = true;
        } else if (staging && own[j] == blk) {  // staged sink/recent token: fp32 values
          const long long base = ((long long)(stage_row_of(p, req, p_first + i, blk) * kPage + j) * p.Hk + hk) * kD + d0;
          const float4* kf = reinterpret_cast<const float4*>(p.stage_k + base);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 a = __ldg(kf + 2 * c), b = __ldg(kf + 2 * c + 1);
            *reinterpret_cast<uint4*>(ks + mma::swz(my_tok, c0 + c)) =
                make_uint4(mma::h2_u32(a.x, a.y), mma::h2_u32(a.z, a.w), mma::h2_u32(b.x, b.y), mma::h2_u32(b.z, b.w));
          }
          par = make_float4(1.f, 0.f, 1.f, 0.f);
          value_tok = true;
        } else {  // INT2 K codes: 64 dims = 16 bytes
          const int cb = kD / 4;
          const uint4 kw = *reinterpret_cast<const uint4*>(pg + j * cb + ((my_q ^ ((j >> 1) & 3)) << 4));
          const uint32_t kk[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t h0[4], h1[4];
            mma::codes8_to_h2(kk[q], h0);
            mma::codes8_to_h2(kk[q] >> 8, h1);
            *reinterpret_cast<uint4*>(ks + mma::swz(my_tok, c0 + 2 * q)) = make_uint4(h0[0], h0[1], h0[2], h0[3]);
            *reinterpret_cast<uint4*>(ks + mma::swz(my_tok, c0 + 2 * q + 1)) = make_uint4(h1[0], h1[1], h1[2], h1[3]);
          }
          if (my_q == 0) {
            const __half* meta = reinterpret_cast<const __half*>(pg + 2 * kPage * cb);
            par = make_float4(__half2float(meta[j]), __half2float(meta[kPage + j]),
                              __half2float(meta[2 * kPage + j]), __half2float(meta[3 * kPage + j]));
          }
        }
        if (my_q == 0) tokp[my_tok] = par;
        // V^T tile: thread = dim, 64 tokens of codes (16 bytes of the dim-major V rows)
        {
          const int d = tid;
          const uint4 vw = *reinterpret_cast<const uint4*>(pg + kPage * (kD / 4) + d * (kPage / 4) + half * 16);
          const uint32_t vv[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t h0[4], h1[4];
            mma::codes8_to_h2(vv[q], h0);
            mma::codes8_to_h2(vv[q] >> 8, h1);
            *reinterpret_cast<uint4*>(vs + swz_vt(d, 2 * q)) = make_uint4(h0[0], h0[1], h0[2], h0[3]);
            *reinterpret_cast<uint4*>(vs + swz_vt(d, 2 * q + 1)) = make_uint4(h1[0], h1[1], h1[2], h1[3]);
          }
        }
        // tokens that carry values instead of codes: overwrite their V^T columns
        if (__syncthreads_or(value_tok)) {
          const int d = tid;
          for (int jj = 0; jj < kTile; ++jj) {
            const int jp = half * kTile + jj, ps = page_pos + jp;
            if (ps >= kv_stop || ps < kv_begin) continue;
            float v;
            if (ps >= prefix) {
              v = __half2float(p.v_fresh[((long long)(q0 + ps - prefix) * p.Hk + hk) * kD + d]);
            } else if (staging && own[jp] == blk) {
              v = __ldg(p.stage_v + ((long long)stage_row_of(p, req, p_first + i, blk) * p.Hk + hk) * kD * kPage +
                        (long long)d * kPage + jp);
            } else {
              continue;
            }
            *reinterpret_cast<__half*>(vs + swz_vt(d, jj >> 3) + (jj & 7) * 2) = __float2half_rn(v);
          }
        }
      }
      __syncthreads();
      // the ring slot is consumed once both tiles of the page are built
      if (half == 1 || tile0 + kTile >= kv_stop) {
        if (tid == 0 && i + kRing < n_pages) issue(i + kRing);
      }
      if (mma_warp) {
        if (four_rt)
          warp_tile<32>(qs_a, ks_a, vs_a, tokp, rt * 16, tok0, tile0, kv_begin, kv_stop, lim_a, lim_b, sq_a, sq_b, sl2,
                        m_a, m_b, l_a, l_b, z_a, z_b, o);
        else
          warp_tile<16>(qs_a, ks_a, vs_a, tokp, rt * 16, tok0, tile0, kv_begin, kv_stop, lim_a, lim_b, sq_a, sq_b, sl2,
                        m_a, m_b, l_a, l_b, z_a, z_b, o);
      }
      __syncthreads();  // tiles are rebuilt next
    }
  }

  // drain: every copy issued must land before the CTA exits (bounded)
  if (tid == 0 && !ok) {
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0; i < n_pages; ++i)
      while (!sm100::mbar_try_wait(&full[i % kRing], (i / kRing) & 1))
        if (globaltimer_ns() - t0 > 200000000ull) break;
  }
  __syncthreads();

  // ---- merge the token-group states of every row tile in shared memory ----
  // per warp: O [16 rows][256] fp32 (16 KB), then m, l, z per row
  float* mo = reinterpret_cast<float*>(smem);  // 8 warps x 16 KB = 128 KB (ring + tiles are dead)
  float* mstat = reinterpret_cast<float*>(smem + 8 * 16384);  // [8 warps][16 rows][3]
#pragma unroll
  for (int o2 = 1; o2 <= 2; o2 <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o2);
    z_a += __shfl_xor_sync(0xffffffffu, z_a, o2);
    z_b += __shfl_xor_sync(0xffffffffu, z_b, o2);
  }
  if (mma_warp) {
    float* wo = mo + warp * 16 * kD;
    const int la = lane >> 2, lb = la + 8;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int d = j * 8 + 2 * (lane & 3);
      *reinterpret_cast<float2*>(wo + la * kD + d) = make_float2(o[j][0], o[j][1]);
      *reinterpret_cast<float2*>(wo + lb * kD + d) = make_float2(o[j][2], o[j][3]);
    }
    if ((lane & 3) == 0) {
      float* ms = mstat + warp * 48;
      ms[la * 3 + 0] = m_a; ms[la * 3 + 1] = l_a; ms[la * 3 + 2] = z_a;
      ms[lb * 3 + 0] = m_b; ms[lb * 3 + 1] = l_b; ms[lb * 3 + 2] = z_b;
    }
  }
  __syncthreads();
  // thread per (row, 32-dim chunk) of the block's rows
  const int n_tg = four_rt ? 2 : 4;
  float* po = p.part_o + ((long long)item * p.Hk + hk) * kRows * kD;
  float* pl = p.part_lse + ((long long)item * p.Hk + hk) * kRows;
  for (int idx = tid; idx < kRows * 8; idx += kThreads) {
    const int r = idx >> 3, chunk = idx & 7;
    const int rtile = r >> 4, rr = r & 15;
    float M = -INFINITY;
    int wl[4];
    for (int t = 0; t < n_tg; ++t) {
      wl[t] = four_rt ? (t * 4 + rtile) : (t * 2 + rtile);
      if (rtile < n_rt) M = fmaxf(M, mstat[wl[t] * 48 + rr * 3]);
    }
    float L = 0.f, acc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) acc[e] = 0.f;
    if (rtile < n_rt && M > -INFINITY) {
      for (int t = 0; t < n_tg; ++t) {
        const float* ms = mstat + wl[t] * 48 + rr * 3;
        const float wgt = exp2f(ms[0] - M);
        L += wgt * ms[1];
        const float zz = ms[2];
        const float* src = mo + wl[t] * 16 * kD + rr * kD + chunk * 32;
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] = fmaf(wgt, src[e] + zz, acc[e]);
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    float* dst = po + r * kD + chunk * 32;
#pragma unroll
    for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(acc[e] * inv, acc[e + 1] * inv, acc[e + 2] * inv, acc[e + 3] * inv);
    if (chunk == 0) pl[r] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
  }
}

}  // namespace
}  // namespace oscar

extern "C" int oscar_int2_attention(const oscar::AttnParams* params, cudaStream_t stream) {
  using namespace oscar;
  const AttnParams& p = *params;
  if (p.n_work <= 0) return 0;
  if (p.D != kD || p.kv_mode != 0) return -320;
  if (p.page_bytes % 16) return -321;
  const Smem L = smem_layout(p.page_bytes);
  if (L.total > 227 * 1024) return -322;
  OSCAR_RC(ensure_smem(int2_attention_kernel, L.total));
  dim3 grid(p.n_work, p.Hk);
  int2_attention_kernel<<<grid, kThreads, L.total, stream>>>(p);
  return (int)cudaGetLastError();
}
