// INT2 paged attention on the 5th-generation tensor cores (tcgen05 + TMEM), for
// work items of at most 32 query rows: decode (q_len 1, rows = g) and MTP verify
// (q_len 4, rows = 4 g = 24 for the 6:1 GQA of the target model).
//
// One CTA per (work item, KV head), 16 warps with fixed roles:
//   warp 0      streams whole page-heads (17,408 B + 512 B of staging owner tags)
//               into a 4-deep shared-memory ring with plain bulk copies, and owns
//               the TMEM allocation (512 columns);
//   warp 1      one thread issues every tcgen05.mma;
//   warps 2-3   row statistics (below);
//   warps 4-7   "K converters": TMEM lane t.  For page i they widen the 2-bit K codes
//               of token t to exact fp16 (0..3) straight into tensor memory (A operand
//               of S^T = K Q^T, M = 128 tokens, K = 256 dims);
//   warps 12-15 "V converters": TMEM lane t, the dim-major V codes of dims t and t+128
//               (A operand of O^T += V^T P'^T, M = 128 dims, K = 128 tokens), beside
//               the K converters: a warp stores about 45 B per cycle into TMEM, so
//               the page's 128 KB of fp16 operands take two warpgroups;
//   warps 8-11  "softmax": TMEM lane t = token t of the page.  They read the
//               page's N scores of token t from TMEM, apply the per-token INT2
//               scale (q.k = s (q.c + (z/s) sum(q)); the zero-point term comes
//               out of the MMA through one extra K-step whose operands are
//               (z/s) and sum(q), each split into fp16 hi + lo), keep the per-row
//               running maxima in registers, and write P' = p * s_v as fp16 into
//               shared memory in the MN-major layout of the B operand of P.V.
// Operand placement keeps shared-memory traffic small: codes never go through
// shared memory as fp16, only the 2-bit page (bulk copy), Q (once) and P' do.
//
// TMEM columns: [0,256) K codes of two pages (double-buffered, so converting page i+1
// overlaps the score MMAs of page i), [256,384) V^T in two token-half slots of 64
// columns (tokens 0-63 and 64-127 of a page, each 2 dim halves x 32; a slot is refilled
// for the next page while the other half's P.V runs), [384,384+2N) two S^T buffers,
// [448,448+2N) the O^T accumulator (2 halves).
// A kind::f16 MMA of M = 128, K = 16 costs ~136 cycles for any N up to 256 whatever its
// operand sources (bench/tcgen05_rates.py), so at N = 32 it runs at an eighth of the
// tensor rate and a page's 33 MMAs are the kernel's floor (~2.3 us); the buffers exist
// to keep the tensor pipe busy back to back.
//
// Softmax bookkeeping.  A row's running max only moves when some score of the
// page exceeds it by more than 2^8 (the probabilities stay <= 256, well inside
// fp16 after scaling by s_v); then the four softmax warps agree on the new maxima
// and rescale O^T in TMEM (after the previous P.V finished) and their partial
// sums.  Each softmax thread keeps per-row partial sums over the tokens it owns:
// l = sum p and C = sum p z_v; they are reduced across threads once at the end:
//     out[r, d] = (O^T[d, r] + C_r) / l_r,   lse_r = m_r + log2 l_r  (log2 units).
// Tokens that are not INT2 (the current chunk's unquantised k/v and staged
// sink/recent tokens) carry their fp16 values with s = 1, z = 0, which gives the
// reference read semantics (paged_attention.py:136-260) in the same pass.
//
// Every wait is bounded: an expired wait sets a CTA abort flag and a status code;
// the roles that synchronise with named barriers agree on aborting through
// bar.red.or so that none is left waiting, in-flight MMAs and bulk copies are
// drained (bounded) and TMEM is freed before the CTA exits.
#include <climits>

#include "common.cuh"
#include "mma.cuh"
#include "params.h"
#include "sm100.cuh"

namespace oscar {
namespace {

constexpr int kD = 256;
constexpr int kPage = 128;
constexpr int kPartRows = 64;  // row stride of the split-KV partials (shared with the merge)
constexpr int kRing = 4;
constexpr int kThreads = 512;
constexpr int kPageBytes = 17408;
constexpr int kSlot = kPageBytes + kPage * 4;  // page + owner tags
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSlack = 8.f;
constexpr uint64_t kBudgetNs = 2000000000ull;
// K codes double-buffered (two pages of 128 columns), one V^T page, two S^T buffers, O^T
constexpr uint32_t kColK = 0, kColV = 256, kColS = 384, kColO = 448, kTmemCols = 512;
constexpr int kBarSoft = 1, kBarStats = 3;
// Initial running maximum: finite, so that exp2(s - m) needs no special case for rows
// without a visible key yet (their scores are -inf), and any visible score moves it.
constexpr float kNoMax = -1e30f;
// The zero-point term z (q . 1) of a code token is folded into the S MMA as
// (z / s) * sum(q) when |z / s| stays well inside fp16; other tokens keep it in the softmax.
constexpr float kZsMax = 16384.f;

OSCAR_DEVICE uint32_t pack_h2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// z / s of a code token, or 0 when its zero-point is not folded (s == 0, |z / s| too big)
OSCAR_DEVICE float folded_zs(float ks, float kz) {
  const float r = ks != 0.f ? kz / ks : 0.f;
  return fabsf(r) <= kZsMax ? r : 0.f;
}
OSCAR_DEVICE bool zs_folded(float ks, float kz) { return ks != 0.f && fabsf(kz / ks) <= kZsMax; }

// Optional per-CTA event timeline (globaltimer ns) for performance analysis; off
// unless a buffer was installed with oscar_attn_tc_trace (slot layout: 128 u64 per CTA).
__device__ unsigned long long* g_tc_trace = nullptr;
constexpr int kTraceSlots = 128;
// The trace buffer pointer is read once per CTA (kernel start) so that a trace point costs
// a timer read and a store, not a global load.
OSCAR_DEVICE void trace(unsigned long long* t, int ev) {
  if (t != nullptr && ev < kTraceSlots)
    t[((long long)blockIdx.y * gridDim.x + blockIdx.x) * kTraceSlots + ev] = globaltimer_ns();
}
// Raw value into a trace slot (e.g. a clock64 difference).
OSCAR_DEVICE void trace_val(unsigned long long* t, int ev, unsigned long long v) {
  if (t != nullptr && ev < kTraceSlots) t[((long long)blockIdx.y * gridDim.x + blockIdx.x) * kTraceSlots + ev] = v;
}
OSCAR_DEVICE unsigned long long clock_dep(float dep) {
  unsigned long long v;
  asm volatile("{\n\t.reg .f32 d;\n\tmov.f32 d, %1;\n\tmov.u64 %0, %%clock64;\n\t}" : "=l"(v) : "f"(dep));
  return v;
}
// Same, ordered after the computation of `dep` (the timer read consumes it).
OSCAR_DEVICE void trace_dep(unsigned long long* t, int ev, float dep) {
  if (t != nullptr && ev < kTraceSlots) {
    uint64_t v;
    asm volatile("{\n\t.reg .f32 d;\n\tmov.f32 d, %1;\n\tmov.u64 %0, %%globaltimer;\n\t}" : "=l"(v) : "f"(dep));
    t[((long long)blockIdx.y * gridDim.x + blockIdx.x) * kTraceSlots + ev] = v;
  }
}

// ---- out-of-line rare paths.  Pages holding value tokens (the current chunk, staged
// sink/recent tokens) are a few per request; their merge code is kept out of the
// per-page loop so the common path of every role stays resident in the
// instruction cache (the whole kernel is larger than it).

// 32 fp16 pairs of 64 K codes (one 16-byte chunk of a token's codes).
OSCAR_DEVICE void k_chunk_codes(const uint8_t* pg, int j, int c, uint32_t (&r)[32]) {
  const uint4 cw = *reinterpret_cast<const uint4*>(pg + j * 64 + ((c ^ ((j >> 1) & 3)) << 4));
  const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t a4[4], b4[4];
    mma::codes8_to_h2(wd[q], a4);
    mma::codes8_to_h2(wd[q] >> 8, b4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      r[8 * q + e] = a4[e];
      r[8 * q + 4 + e] = b4[e];
    }
  }
}

// K row of a warp in which some token carries values: lane j writes fp16 values
// (kind 1: fresh fp16 row `kf`, kind 2: staged fp32 row `sk`) or its codes.
__device__ __noinline__ void k_row_mixed(uint32_t taddr, const uint8_t* pg, int j, int kind, const __half* kf,
                                         const float* sk) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    if (kind == 1) {
      const uint4* src = reinterpret_cast<const uint4*>(kf + 64 * c);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint4 v = __ldg(src + q);
        r[4 * q] = v.x;
        r[4 * q + 1] = v.y;
        r[4 * q + 2] = v.z;
        r[4 * q + 3] = v.w;
      }
    } else if (kind == 2) {
      const float4* src = reinterpret_cast<const float4*>(sk + 64 * c);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const float4 v = __ldg(src + q);
        r[2 * q] = mma::h2_u32(v.x, v.y);
        r[2 * q + 1] = mma::h2_u32(v.z, v.w);
      }
    } else {
      k_chunk_codes(pg, j, c, r);
    }
    sm100::tmem_st_32x32b_x32(taddr + 32 * c, r);
  }
}

// 64 tokens of V^T row d (one page half) when some of them carry values: staged
// tokens (mask sm, from the dim-major staging row `srow`, may be null when sm == 0)
// and current-chunk tokens without a staging seat (mask fm, fp16 from the fresh
// buffer: token tl at vf[fbase + tl * fstride]).  Codes elsewhere.
__device__ __noinline__ void v_half_mixed(uint32_t taddr, uint4 cw, uint64_t sm, uint64_t fm, const float* srow,
                                          const __half* vf, long long fbase, long long fstride) {
  uint32_t r[32];
  const uint32_t w4[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t x4[4], y4[4];
    mma::codes8_to_h2(w4[q], x4);
    mma::codes8_to_h2(w4[q] >> 8, y4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      r[8 * q + e] = x4[e];
      r[8 * q + 4 + e] = y4[e];
    }
  }
  if (sm != 0ull) {
    const float4* s4 = reinterpret_cast<const float4*>(srow);
#pragma unroll 8
    for (int q = 0; q < 16; ++q) {
      const float4 v = __ldg(s4 + q);
      const uint32_t lo = mma::h2_u32(v.x, v.y), hi = mma::h2_u32(v.z, v.w);
      const uint32_t m = (uint32_t)(sm >> (4 * q)) & 15u;  // tokens 4q .. 4q + 3
      const uint32_t k0 = ((m & 1u) ? 0u : 0x0000ffffu) | ((m & 2u) ? 0u : 0xffff0000u);
      const uint32_t k1 = ((m & 4u) ? 0u : 0x0000ffffu) | ((m & 8u) ? 0u : 0xffff0000u);
      r[2 * q] = (r[2 * q] & k0) | (lo & ~k0);
      r[2 * q + 1] = (r[2 * q + 1] & k1) | (hi & ~k1);
    }
  }
  while (fm != 0ull) {
    const int tl = __ffsll((long long)fm) - 1;
    fm &= fm - 1ull;
    const uint32_t hv = (uint32_t)__half_as_ushort(vf[fbase + (long long)tl * fstride]);
    const int k = tl >> 1;
#pragma unroll
    for (int kk = 0; kk < 32; ++kk)
      if (kk == k) r[kk] = (tl & 1) ? ((r[kk] & 0x0000ffffu) | (hv << 16)) : ((r[kk] & 0xffff0000u) | hv);
  }
  sm100::tmem_st_32x32b_x32(taddr, r);
}

// O^T (both halves, N columns each) scaled by alpha[r] per row column r.
template <int N>
OSCAR_DEVICE void rescale_o(uint32_t taddr, const float* alpha) {
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    uint32_t o[N];
    if constexpr (N == 32)
      sm100::tmem_ld_32x32b_x32(taddr + h * N, o);
    else
      sm100::tmem_ld_32x32b_x16(taddr + h * N, o);
    sm100::tmem_ld_wait();
#pragma unroll
    for (int r = 0; r < N; ++r) o[r] = __float_as_uint(__uint_as_float(o[r]) * alpha[r]);
    if constexpr (N == 32)
      sm100::tmem_st_32x32b_x32(taddr + h * N, o);
    else
      sm100::tmem_st_32x32b_x16(taddr + h * N, o);
  }
  sm100::tmem_st_wait();
}

template <int N>
struct TcLayout {
  static constexpr int kQOff = kRing * kSlot;  // 71,680: 1024-aligned
  static constexpr int kQBytes = N * 512;       // 4 chunks of 64 dims x N rows x 128 B
  // zero-point step of S^T = K Q^T, K-major with the 32-byte swizzle (one K-step of 16):
  // Q side [N rows][sum(q) hi, lo, hi, 0...], K side [128 tokens][z' hi, hi, lo, 0...]
  static constexpr int kQzOff = kQOff + kQBytes;
  static constexpr int kZaOff = kQzOff + N * 32;
  static constexpr int kPOff = kZaOff + 2 * kPage * 32;
  static constexpr int kPBytes = kPage * N * 2;  // one P' buffer: 128 tokens x N fp16
  static constexpr int kMisc = kPOff + 2 * kPBytes;
  static constexpr int kSq = kMisc;                  // N floats: sum(q) per row
  static constexpr int kLim = kSq + N * 4;           // N ints: last visible key position per row
  static constexpr int kMsm = kLim + N * 4;          // N floats: running row maxima (log2 units)
  static constexpr int kRed = kMsm + N * 4;          // N x 4 floats: per-warp page maxima
  static constexpr int kAlpha = kRed + N * 16;       // 2 x N floats: rescale factor of a page
  static constexpr int kFin = kAlpha + 2 * N * 4;    // groups x 2N floats: partial l, C
  static constexpr int kCoef = kFin + 1024;          // 2 x 128 float2: (1/s_v, z_v/s_v)
  static constexpr int kVmask = kCoef + 2 * kPage * 8;  // 2 x 4 u32
  static constexpr int kUpd = kVmask + 32;           // 2 ints + resc flag
  static constexpr int kSlotBlk = kUpd + 16;         // kRing ints
  static constexpr int kTmemSlot = kSlotBlk + kRing * 4;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kBars = (kAbort + 4 + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * kRing + 2 * 8 + 2;
  static constexpr int kTotal = kBars + kNumBars * 8;
  // at least half the SM's shared memory: one CTA per SM (it holds all 512 TMEM columns)
  static constexpr int kAlloc = (kTotal > 120 * 1024 ? kTotal : 120 * 1024) + 1024;  // + base alignment
};

struct Bars {
  uint64_t* raw_full;   // [kRing]
  uint64_t* raw_empty;  // [kRing]
  uint64_t* k_full;     // [2]
  uint64_t* k_empty;    // [2]
  uint64_t* v_full;     // [2] token halves of the V page
  uint64_t* v_empty;    // [2]
  uint64_t* s_full;   // [2]
  uint64_t* s_empty;  // [2]
  uint64_t* p_full;   // [2]
  uint64_t* p_empty;  // [2]
  uint64_t* mma_done;
  uint64_t* stats_done;
};

// Transposed butterfly: on return lane r holds the reduction of row r (N = 32) or
// of row r % 16 (N = 16) over the 32 lanes; v[] is clobbered.
template <int N, bool kMax>
OSCAR_DEVICE float rows_reduce(float (&v)[N]) {
  const int lane = threadIdx.x & 31;
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
  if constexpr (N == 16) {
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = op(v[k], __shfl_xor_sync(0xffffffffu, v[k], 16));
  }
  constexpr int kFirst = N == 32 ? 16 : 8;
#pragma unroll
  for (int o = kFirst; o >= 1; o >>= 1) {
    const bool up = lane & o;
#pragma unroll
    for (int k = 0; k < o; ++k) {
      const float send = up ? v[k] : v[k + o];
      const float keep = up ? v[k + o] : v[k];
      v[k] = op(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return v[0];
}

template <int N>
__global__ void __launch_bounds__(kThreads, 1) int2_attention_tc_kernel(AttnParams p) {
  unsigned long long* const tr = g_tc_trace;  // per-CTA copy of the trace buffer pointer
  using L = TcLayout<N>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // swizzled operand tiles need 1024-byte aligned shared addresses
  uint8_t* smem = smem_raw + ((1024u - (sm100::smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  uint8_t* qs = smem + L::kQOff;
  uint8_t* qz = smem + L::kQzOff;
  uint8_t* za = smem + L::kZaOff;
  uint8_t* ps = smem + L::kPOff;
  float* sq = reinterpret_cast<float*>(smem + L::kSq);
  int* lim = reinterpret_cast<int*>(smem + L::kLim);
  float* msm = reinterpret_cast<float*>(smem + L::kMsm);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* alpha = reinterpret_cast<float*>(smem + L::kAlpha);
  float* fin = reinterpret_cast<float*>(smem + L::kFin);
  float2* coef = reinterpret_cast<float2*>(smem + L::kCoef);
  uint32_t* vmask = reinterpret_cast<uint32_t*>(smem + L::kVmask);
  volatile int* upd = reinterpret_cast<volatile int*>(smem + L::kUpd);
  volatile int* resc_flag = reinterpret_cast<volatile int*>(smem + L::kUpd + 8);
  int* slot_blk = reinterpret_cast<int*>(smem + L::kSlotBlk);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBars);
  Bars B{bar, bar + kRing, bar + 2 * kRing, bar + 2 * kRing + 2, bar + 2 * kRing + 4, bar + 2 * kRing + 6,
         bar + 2 * kRing + 8, bar + 2 * kRing + 10, bar + 2 * kRing + 12, bar + 2 * kRing + 14, bar + 2 * kRing + 16,
         bar + 2 * kRing + 17};

  const int item = blockIdx.x, hk = blockIdx.y;
  const int4 w = p.work[item];
  const int req = w.x, row0 = w.y, kv_begin = w.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.Hq / p.Hk;
  const int q0 = p.q_start[req];
  const int qlen = p.q_start[req + 1] - q0;
  const int prefix = p.seq_lens[req] - qlen;
  const int* bt = p.block_tables + (long long)req * p.bt_stride;
  const int nrows = max(0, min(N, qlen * g - row0));
  const int kv_stop = min(w.w, nrows > 0 ? prefix + (row0 + nrows - 1) / g + 1 : 0);
  const bool staging = p.stage_rows > 0;
  const int p_first = kv_begin / kPage;
  const int n_pages = kv_stop > kv_begin ? (kv_stop - 1) / kPage - p_first + 1 : 0;

  // ---------------------------------------------------------------- setup
  if (tid == 0) trace(tr, 0);
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, kTmemCols);
    sm100::tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < L::kNumBars; ++i) sm100::mbar_init(&bar[i], 1);
    for (int s = 0; s < kRing; ++s) sm100::mbar_init(&B.raw_empty[s], 14);  // 4 + 4 converter, 4 softmax, 2 stats warps
    for (int b = 0; b < 2; ++b) sm100::mbar_init(&B.p_empty[b], 3);       // P.V commit + 2 stats warps
    sm100::mbar_init(B.stats_done, 2);
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&B.v_full[b], 4);
      sm100::mbar_init(&B.k_full[b], 4);
      sm100::mbar_init(&B.s_empty[b], 4);
      sm100::mbar_init(&B.p_full[b], 4);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  // Q tile, K-major with the 128-byte swizzle: [dim chunk of 64][row][128 B]
  for (int idx = tid; idx < N * 32; idx += kThreads) {
    const int r = idx >> 5, ch = idx & 31;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows) {
      const int gr = row0 + r, t = gr / g, h = gr % g;
      v = __ldg(reinterpret_cast<const uint4*>(p.q + ((long long)(q0 + t) * p.Hq + hk * g + h) * kD) + ch);
    }
    *reinterpret_cast<uint4*>(qs + (ch >> 3) * (N * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)) = v;
  }
  __syncthreads();
  if (tid < N) {
    float acc = 0.f;
    for (int ch = 0; ch < 32; ++ch) {
      const uint4 v = *reinterpret_cast<const uint4*>(qs + (ch >> 3) * (N * 128) + tid * 128 + (((ch & 7) ^ (tid & 7)) << 4));
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        acc += f.x + f.y;
      }
    }
    sq[tid] = acc;
    lim[tid] = tid < nrows ? prefix + (row0 + tid) / g : -1;
    msm[tid] = kNoMax;
    const __half hi = __float2half_rn(acc), lo = __float2half_rn(acc - __half2float(hi));
    const uint32_t w0 = pack_h2(hi, lo), w1 = pack_h2(hi, __float2half_rn(0.f));
    const int sw = (tid >> 2) & 1;
    *reinterpret_cast<uint4*>(qz + tid * 32 + (sw << 4)) = make_uint4(w0, w1, 0u, 0u);
    *reinterpret_cast<uint4*>(qz + tid * 32 + ((sw ^ 1) << 4)) = make_uint4(0u, 0u, 0u, 0u);
  }
  for (int idx = tid; idx < 2 * kPage * 2; idx += kThreads)
    *reinterpret_cast<uint4*>(za + idx * 16) = make_uint4(0u, 0u, 0u, 0u);
  sm100::fence_proxy_async();  // Q tile: generic writes -> tensor-core reads
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (tid == 0) trace(tr, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ page producer
    if (lane == 0) {
      const uint32_t tx = kPageBytes + (staging ? kPage * 4 : 0);
      int issued = 0;
      for (int i = 0; i < n_pages; ++i) {
        const int s = i % kRing;
        if (i >= kRing && !sm100::mbar_wait_sleep(&B.raw_empty[s], ((i / kRing) - 1) & 1, abort_flag, p.status,
                                            kTimeoutSlotEmpty, kBudgetNs))
          break;
        const int blk = bt[p_first + i];
        slot_blk[s] = blk;
        uint8_t* dst = ring + s * kSlot;
        sm100::mbar_arrive_expect_tx(&B.raw_full[s], tx);
        sm100::bulk_load(dst, p.pool + ((long long)blk * p.Hk + hk) * kPageBytes, kPageBytes, &B.raw_full[s]);
        if (staging)
          sm100::bulk_load(dst + kPageBytes, p.owner + (long long)stage_row_of(p, req, p_first + i, blk) * kPage, kPage * 4,
                           &B.raw_full[s]);
        issued = i + 1;
        if (i < 8) trace(tr, 8 + i);
      }
      if (*abort_flag) {  // copies in flight must land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        for (int i = max(0, issued - kRing); i < issued; ++i)
          while (!sm100::mbar_try_wait(&B.raw_full[i % kRing], (i / kRing) & 1))
            if (globaltimer_ns() - t0 > 200000000ull) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idq = sm100::idesc_f16(128, N, false, false);
      const uint32_t idp = sm100::idesc_f16(128, N, false, true);
      const uint32_t qa = sm100::smem_addr(qs), pa = sm100::smem_addr(ps);
      const uint64_t zad = sm100::smem_desc(sm100::smem_addr(za), 16, 256, 6);
      const uint64_t qzd = sm100::smem_desc(sm100::smem_addr(qz), 16, 256, 6);
      constexpr uint32_t kPLayout = N == 32 ? 4u : 6u;  // P' rows of N fp16: 64 B / 32 B swizzle
      constexpr uint32_t kPAtom = 8 * N * 2;           // 8 tokens
      // P.V of page j, one token half (one V slot) at a time: the V converters refill
      // a slot while the other half's MMAs run
      auto pv = [&](int j) -> bool {
        if (!sm100::mbar_wait_sleep(&B.p_full[j & 1], (j >> 1) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs))
          return false;
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          if (!sm100::mbar_wait_sleep(&B.v_full[hf], j & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs))
            return false;
          sm100::tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t bd = sm100::smem_desc(pa + (j & 1) * L::kPBytes + (hf * 4 + ks) * 2 * kPAtom, 16, kPAtom,
                                                   kPLayout);
              sm100::umma_f16_tmem_a(tbase + kColO + h * N, tbase + kColV + hf * 64 + h * 32 + ks * 8, bd, idp,
                                     (j > 0 || hf > 0 || ks > 0) ? 1u : 0u);
            }
          sm100::umma_commit(&B.v_empty[hf]);
        }
        sm100::umma_commit(&B.p_empty[j & 1]);
        return true;
      };
      bool ok = true;
      for (int i = 0; i < n_pages && ok; ++i) {
        if (!sm100::mbar_wait_sleep(&B.k_full[i & 1], (i >> 1) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs)) {
          ok = false;
          break;
        }
        if (i < 4) trace(tr, 88 + i);
        if (i >= 2 && !sm100::mbar_wait_sleep(&B.s_empty[i & 1], ((i >> 1) - 1) & 1, abort_flag, p.status,
                                        kTimeoutAccEmpty, kBudgetNs)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const unsigned long long mc0 = (tr != nullptr) ? clock64() : 0ull;
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint64_t qd = sm100::smem_desc(qa + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024, 2);
          sm100::umma_f16_tmem_a(tbase + kColS + (i & 1) * N, tbase + kColK + (i & 1) * 128 + kk * 8, qd, idq,
                                 kk > 0 ? 1u : 0u);
        }
        // + (z/s) sum(q): K-side and Q-side tiles in shared memory, 32-byte swizzle
        sm100::umma_bf16(tbase + kColS + (i & 1) * N, zad + (uint64_t)(((i & 1) * kPage * 32) >> 4), qzd, idq, 1u);
        if (i < 4 && tr != nullptr) trace_val(tr, 112 + i, clock64() - mc0);
        sm100::umma_commit(&B.s_full[i & 1]);
        if (i < 8) trace(tr, 16 + i);
        sm100::umma_commit(&B.k_empty[i & 1]);
        if (i >= 1) ok = pv(i - 1);
      }
      if (ok && n_pages > 0) pv(n_pages - 1);
      // nothing may still write TMEM when it is freed
      sm100::umma_commit(B.mma_done);
      const uint64_t t0 = globaltimer_ns();
      while (!sm100::mbar_try_wait(B.mma_done, 0))
        if (globaltimer_ns() - t0 > 200000000ull) break;
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ K converters
    const int ct = tid - 128;  // TMEM lane
    const uint32_t lrow = (uint32_t)(ct & ~31) << 16;
    // No named barriers in the converter loops: every warp arrives on the mbarriers
    // itself, so a warp whose bounded wait expires simply leaves (the others time out
    // in turn).  K of page i goes to TMEM slot i & 1, free once S(i - 2) is done.
    for (int i = 0; i < n_pages; ++i) {
        const int s = i % kRing;
        if (!sm100::mbar_wait_sleep(&B.raw_full[s], (i / kRing) & 1, abort_flag, p.status, kTimeoutTmaFull,
                                    kBudgetNs))
          break;
        if (i >= 2 && !sm100::mbar_wait_sleep(&B.k_empty[i & 1], ((i >> 1) - 1) & 1, abort_flag, p.status,
                                              kTimeoutAccEmpty, kBudgetNs))
          break;
        const uint32_t kcol = kColK + (i & 1) * 128;
        uint8_t* zrow = za + (i & 1) * kPage * 32;
        if (ct == 0 && i < 4) trace(tr, 84 + i);
        const unsigned long long kc0 = (tr != nullptr) ? clock64() : 0ull;
        const uint8_t* pg = ring + s * kSlot;
        const int* own = reinterpret_cast<const int*>(pg + kPageBytes);
        const int blk = slot_blk[s];
        const int page_pos = (p_first + i) * kPage;
        sm100::tc_fence_after();
        {
          // K codes of token ct -> 128 columns of fp16 pairs
          const int j = ct, pos = page_pos + j;
          const bool in = pos >= kv_begin && pos < kv_stop;
          const bool stg_j = in && staging && own[j] == blk;
          const int kind = !in ? 0 : stg_j ? 2 : pos >= prefix ? 1 : 3;
          {
            // zero-point row of token j for the S MMA's extra K-step: (z/s hi, z/s hi, z/s lo)
            // against (sum(q) hi, lo, hi) on the Q side
            const __half* meta = reinterpret_cast<const __half*>(pg + 2 * kPage * 64);
            const float zs = kind == 3 ? folded_zs(__half2float(meta[j]), __half2float(meta[kPage + j])) : 0.f;
            const __half zh = __float2half_rn(zs), zl = __float2half_rn(zs - __half2float(zh));
            *reinterpret_cast<uint4*>(zrow + j * 32 + (((j >> 2) & 1) << 4)) =
                make_uint4(pack_h2(zh, zh), pack_h2(zl, __float2half_rn(0.f)), 0u, 0u);
          }
          if (__any_sync(0xffffffffu, kind == 1 || kind == 2)) {
            const __half* kf = kind == 1 ? p.k_fresh + ((long long)(q0 + pos - prefix) * p.Hk + hk) * kD : nullptr;
            const float* sk = kind == 2 ? p.stage_k + ((long long)(stage_row_of(p, req, p_first + i, blk) * kPage + j) *
                                                           p.Hk + hk) * kD
                                        : nullptr;
            k_row_mixed(tbase + lrow + kcol, pg, j, kind, kf, sk);
          } else {
            // out-of-range tokens keep their (finite) codes: their scores are masked
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              k_chunk_codes(pg, j, c, r);
              sm100::tmem_st_32x32b_x32(tbase + lrow + kcol + 32 * c, r);
            }
          }
          const unsigned long long kc1 = (tr != nullptr) ? clock64() : 0ull;
          sm100::tmem_st_wait();
          sm100::tc_fence_before();
          if (ct == 0 && i < 4) {
            const unsigned long long kc2 = clock64();
            trace_val(tr, 96 + i, kc1 - kc0);
            trace_val(tr, 100 + i, kc2 - kc1);
          }
        }
        sm100::fence_proxy_async();  // zero-point row: generic write -> tensor-core read
        __syncwarp();
        if (lane == 0) {
          sm100::mbar_arrive(&B.k_full[i & 1]);
          sm100::mbar_arrive(&B.raw_empty[s]);
        }
        if (ct == 0 && i < 8) trace(tr, 24 + i);
          }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ V converters
    // V^T of page i into the two token-half slots, each free once P.V(i - 1) of that
    // half is done; they run beside the K converters, so a page's two conversions overlap.
    const int ct = tid - 384;  // TMEM lane
    const uint32_t lrow = (uint32_t)(ct & ~31) << 16;
    uint32_t smk[4], fmk[4];  // value-token masks of the page
    for (int i = 0; i < n_pages; ++i) {
        // V^T of page i, dims ct and ct + 128 -> 2 x 64 columns
        const int s = i % kRing;
        if (!sm100::mbar_wait_sleep(&B.raw_full[s], (i / kRing) & 1, abort_flag, p.status, kTimeoutTmaFull,
                                    kBudgetNs))
          break;
        const uint8_t* pg = ring + s * kSlot;
        const int* own = reinterpret_cast<const int*>(pg + kPageBytes);
        const int blk = slot_blk[s];
        const int page_pos = (p_first + i) * kPage;
        // Tokens that carry values, as 128-bit masks computed by every warp for itself
        // (lane l looks at tokens l, 32 + l, 64 + l, 96 + l): staged sink/recent tokens
        // (owner tag == block, read from the staging arena; this includes current-chunk
        // tokens that were staged in this step - the same values) and current-chunk
        // tokens that are not staged (read from the fresh buffer).
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int tj = 32 * q + lane, ps_ = page_pos + tj;
          const bool in = ps_ >= kv_begin && ps_ < kv_stop;
          const bool stg = in && staging && own[tj] == blk;
          const bool frs = in && !stg && ps_ >= prefix;
          smk[q] = __ballot_sync(0xffffffffu, stg);
          fmk[q] = __ballot_sync(0xffffffffu, frs);
        }
        bool vok = true;
#pragma unroll 1
        for (int hf = 0; hf < 2 && vok; ++hf) {
          // slot hf holds tokens 64 hf .. 64 hf + 63 of the page; free once P.V(i - 1) of
          // that half is done
          if (i >= 1 && !sm100::mbar_wait_sleep(&B.v_empty[hf], (i - 1) & 1, abort_flag, p.status, kTimeoutAccEmpty,
                                                kBudgetNs)) {
            vok = false;
            break;
          }
          if (ct == 0 && i < 4 && hf == 0) trace(tr, 92 + i);
          const unsigned long long vc0 = (tr != nullptr) ? clock64() : 0ull;
          sm100::tc_fence_after();
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            const int d = ct + 128 * h;
            const uint4 cw = reinterpret_cast<const uint4*>(pg + kPage * 64 + d * 32)[hf];
            const uint32_t taddr = tbase + lrow + kColV + hf * 64 + h * 32;
            const uint64_t sm = hf ? ((uint64_t)smk[3] << 32) | smk[2] : ((uint64_t)smk[1] << 32) | smk[0];
            const uint64_t fm = hf ? ((uint64_t)fmk[3] << 32) | fmk[2] : ((uint64_t)fmk[1] << 32) | fmk[0];
            if ((sm | fm) != 0ull) {
              // staged tokens: this dim's 64 values of the page half are contiguous fp32
              // in the dim-major staging arena
              const float* srow = sm != 0ull ? p.stage_v +
                                                   ((long long)stage_row_of(p, req, p_first + i, blk) * p.Hk + hk) *
                                                       kD * kPage +
                                                   (long long)d * kPage + hf * 64
                                             : nullptr;
              const long long fbase = ((long long)(q0 + page_pos + hf * 64 - prefix) * p.Hk + hk) * kD + d;
              v_half_mixed(taddr, cw, sm, fm, srow, p.v_fresh, fbase, (long long)p.Hk * kD);
            } else {
              uint32_t r[32];
              const uint32_t w4[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t x4[4], y4[4];
                mma::codes8_to_h2(w4[q], x4);
                mma::codes8_to_h2(w4[q] >> 8, y4);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  r[8 * q + e] = x4[e];
                  r[8 * q + 4 + e] = y4[e];
                }
              }
              sm100::tmem_st_32x32b_x32(taddr, r);
            }
          }
          if (hf == 1 && ct == 0 && i < 4 && tr != nullptr) trace_val(tr, 104 + i, clock64() - vc0);
          sm100::tmem_st_wait();
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(&B.v_full[hf]);
        }
        if (!vok) break;
        if (ct == 0 && i < 8) trace(tr, 32 + i);
        if (lane == 0) sm100::mbar_arrive(&B.raw_empty[s]);
          }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ row statistics
    // l_r = sum_j p_jr and C_r = sum_j p_jr z_vj, read back from the fp16 P' tile the
    // tensor cores consume (P' = p s_v), so they match the P.V product exactly.
    const int tt = tid - 64;
    constexpr int kPairs = N / 2;             // row pairs
    constexpr int kGroups = 64 / kPairs;      // token groups
    constexpr int kTok = kPage / kGroups;     // tokens per group
    const int rp = tt % kPairs, grp = tt / kPairs;
    float l0 = 0.f, l1 = 0.f, c0 = 0.f, c1 = 0.f;
    bool dead = false, aborted = false;
    for (int i = 0; i < n_pages; ++i) {
      const int s = i % kRing, b = i & 1;
      bool ok = !dead && sm100::mbar_wait_sleep(&B.p_full[b], (i >> 1) & 1, abort_flag, p.status, kTimeoutAccFull,
                                          kBudgetNs);
      if (ok) {
        // per-token coefficients (1/s_v, z_v/s_v) of this page
        const uint8_t* pg = ring + s * kSlot;
        const int* own = reinterpret_cast<const int*>(pg + kPageBytes);
        const int blk = slot_blk[s];
        const __half* meta = reinterpret_cast<const __half*>(pg + 2 * kPage * 64);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = 2 * tt + e, pos = (p_first + i) * kPage + j;
          float2 cf = make_float2(0.f, 0.f);
          if (pos >= kv_begin && pos < kv_stop) {
            if (pos >= prefix || (staging && own[j] == blk)) {
              cf = make_float2(1.f, 0.f);
            } else {
              const float sv = __half2float(meta[2 * kPage + j]);
              const float inv = 1.f / sv;
              cf = make_float2(inv, __half2float(meta[3 * kPage + j]) * inv);
            }
          }
          coef[b * kPage + j] = cf;
        }
      }
      if (sm100::bar_red_or(kBarStats, 64, !ok)) {
        aborted = true;
        break;
      }
      if (upd[b]) {  // the row maxima moved on this page: rescale the running sums
        const float a0 = alpha[b * N + 2 * rp], a1 = alpha[b * N + 2 * rp + 1];
        l0 *= a0;
        c0 *= a0;
        l1 *= a1;
        c1 *= a1;
      }
      const uint8_t* pt = ps + b * L::kPBytes;
#pragma unroll 4
      for (int k = 0; k < kTok; ++k) {
        const int j = grp * kTok + k;
        const int c = (2 * rp) >> 3;
        const int sw = N == 32 ? (c ^ ((j >> 1) & 3)) : (c ^ ((j >> 2) & 1));
        const uint32_t hv = *reinterpret_cast<const uint32_t*>(pt + j * (N * 2) + (sw << 4) + ((2 * rp) & 7) * 2);
        const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(&hv));
        const float2 cf = coef[b * kPage + j];
        l0 = fmaf(pf.x, cf.x, l0);
        c0 = fmaf(pf.x, cf.y, c0);
        l1 = fmaf(pf.y, cf.x, l1);
        c1 = fmaf(pf.y, cf.y, c1);
      }
      __syncwarp();
      if (lane == 0) {
        sm100::mbar_arrive(&B.p_empty[b]);
        sm100::mbar_arrive(&B.raw_empty[s]);
      }
    }
    if (!aborted) {
      float* fs = fin + grp * 2 * N;  // [group][l (N) | C (N)]
      fs[2 * rp] = l0;
      fs[2 * rp + 1] = l1;
      fs[N + 2 * rp] = c0;
      fs[N + 2 * rp + 1] = c1;
    }
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(B.stats_done);
  } else if (warp >= 8 && warp < 12) {
    // ------------------------------------------------------------ softmax
    const int st = tid - 256;  // TMEM lane = token of the page
    const int swarp = st >> 5;
    const uint32_t lrow = (uint32_t)(st & ~31) << 16;
    const float sl2 = p.scale * kLog2e;
    // Running row maxima are read as float4 broadcasts from shared memory (they only
    // change on the rare pages that move a maximum by more than the slack).  sum(q) and
    // the causal limits are needed only for unfolded zero-points and the last pages:
    // lane r holds row r, broadcast by shuffles on those pages.
    const float sq_l = sq[lane % N];
    const int lim_l = lim[lane % N];
    const float4* mr4 = reinterpret_cast<const float4*>(msm);
    bool dead = false, aborted = false;
    for (int i = 0; i < n_pages; ++i) {
      const int s = i % kRing, b = i & 1;
      bool ok = !dead && sm100::mbar_wait_sleep(&B.s_full[b], (i >> 1) & 1, abort_flag, p.status, kTimeoutAccFull,
                                          kBudgetNs);
      if (st == 0 && i < 4) trace(tr, 48 + 4 * i);
      float sc[N];
      if (ok) {
        uint32_t raw[N];
        sm100::tc_fence_after();
        if constexpr (N == 32)
          sm100::tmem_ld_32x32b_x32(tbase + lrow + kColS + b * N, raw);
        else
          sm100::tmem_ld_32x32b_x16(tbase + lrow + kColS + b * N, raw);
        sm100::tmem_ld_wait();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&B.s_empty[b]);
#pragma unroll
        for (int r = 0; r < N; ++r) sc[r] = __uint_as_float(raw[r]);
        ok = sm100::mbar_wait_sleep(&B.raw_full[s], (i / kRing) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs);
      }
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform before the shuffles below
      if (st == 0 && i < 4) trace(tr, 49 + 4 * i);
      float vs = 0.f;
      bool need = false;
      if (ok) {
        const uint8_t* pg = ring + s * kSlot;
        const int* own = reinterpret_cast<const int*>(pg + kPageBytes);
        const int blk = slot_blk[s];
        const int j = st, pos = (p_first + i) * kPage + j;
        const bool in = pos >= kv_begin && pos < kv_stop;
        float ks = 0.f, kz = 0.f;
        if (in) {
          if (pos >= prefix || (staging && own[j] == blk)) {
            ks = 1.f;
            vs = 1.f;
          } else {
            const __half* meta = reinterpret_cast<const __half*>(pg + 2 * kPage * 64);
            ks = __half2float(meta[j]);
            kz = __half2float(meta[kPage + j]);
            vs = __half2float(meta[2 * kPage + j]);
          }
        }
        const bool hist = pos < prefix;
        // zero-point z sum(q) of code tokens comes with S from the MMA (folded) unless
        // |z / s| is too large for fp16 (then it is added here)
        const bool unf = in && !(pos >= prefix || (staging && own[j] == blk)) && !zs_folded(ks, kz);
        if (i < 4) trace_dep(tr, st == 0 ? 64 + 4 * i : kTraceSlots, ks + kz + vs);
        const unsigned long long cl0 = clock_dep(ks + kz + vs);
        const float kss = ks * sl2, kzs = unf ? kz * sl2 : 0.f;
        const bool page_hist = (p_first + i + 1) * kPage <= prefix;
        float dmax = -INFINITY;
        if (page_hist && !__any_sync(0xffffffffu, unf)) {
#pragma unroll
          for (int r = 0; r < N; r += 4) {
            const float4 m4 = mr4[r / 4];
            const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              sc[r + e] = in ? kss * sc[r + e] : -INFINITY;
              dmax = fmaxf(dmax, sc[r + e] - mv[e]);
            }
          }
        } else {
#pragma unroll
          for (int r = 0; r < N; r += 4) {
            const float4 m4 = mr4[r / 4];
            const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float qv = __shfl_sync(0xffffffffu, sq_l, r + e);
              const int lv = page_hist ? INT_MAX : __shfl_sync(0xffffffffu, lim_l, r + e);
              const bool vis = in && (hist || pos <= lv);
              sc[r + e] = vis ? fmaf(kss, sc[r + e], kzs * qv) : -INFINITY;
              dmax = fmaxf(dmax, sc[r + e] - mv[e]);
            }
          }
        }
        need = dmax > kSlack;
        if (i < 4) trace_dep(tr, st == 0 ? 65 + 4 * i : kTraceSlots, sc[N - 1] + (need ? 1.f : 0.f));
        const unsigned long long cl1 = clock_dep(sc[N - 1] + (need ? 1.f : 0.f));
        if (st == 0 && i < 4) trace_val(tr, 80 + i, cl1 - cl0);
      }
      // P' buffer b (and alpha/upd slot b) are free once P.V(i-2) and the stats of page i-2 are done
      if (ok && i >= 2)
        ok = sm100::mbar_wait_sleep(&B.p_empty[b], ((i >> 1) - 1) & 1, abort_flag, p.status, kTimeoutAccEmpty, kBudgetNs);
      if (st == 0 && i < 4) trace(tr, 50 + 4 * i);
      // one barrier on the common path: abort and "a maximum moved" are both rare
      bool upd_now = false;
      if (sm100::bar_red_or(kBarSoft, 128, !ok || need)) {
        if (sm100::bar_red_or(kBarSoft, 128, !ok)) {
          aborted = true;
          break;
        }
        upd_now = true;  // no warp aborted, so some warp saw a maximum move
      }
      if (st == 0 && i < 4) trace(tr, 51 + 4 * i);
      if (upd_now) {
        // agree on the new row maxima
        {
          float t[N];
#pragma unroll
          for (int r = 0; r < N; ++r) t[r] = sc[r];
          const float wm = rows_reduce<N, true>(t);
          if (lane < N) red[lane * 4 + swarp] = wm;
        }
        if (st == 0) *resc_flag = 0;
        sm100::bar_sync(kBarSoft, 128);
        if (st < N) {
          const float4 q4 = *reinterpret_cast<const float4*>(red + st * 4);
          const float pm = fmaxf(fmaxf(q4.x, q4.y), fmaxf(q4.z, q4.w));
          const float mo = msm[st];
          const float mn = fmaxf(mo, pm);
          const float a = (mn == mo) ? 1.f : (mo == -INFINITY ? 0.f : exp2f(mo - mn));
          alpha[b * N + st] = a;
          msm[st] = mn;
          if (a != 1.f) *resc_flag = 1;
        }
        sm100::bar_sync(kBarSoft, 128);
        if (*resc_flag && i > 0) {  // O^T holds pages < i: rescale its columns once P.V(i-1) is done
          bool ok2 = sm100::mbar_wait_sleep(&B.p_empty[(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag, p.status,
                                      kTimeoutAccFull, kBudgetNs);
          if (ok2) {
            sm100::tc_fence_after();
            rescale_o<N>(tbase + lrow + kColO, alpha + b * N);
            sm100::tc_fence_before();
          }
          ok = ok2;
        }
      }
      if (st == 0) upd[b] = upd_now ? 1 : 0;
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        uint32_t pk[N / 2];
#pragma unroll
        for (int r = 0; r < N; r += 4) {
          const float4 m4 = mr4[r / 4];
          pk[r / 2] = mma::h2_u32(exp2f(sc[r] - m4.x) * vs, exp2f(sc[r + 1] - m4.y) * vs);
          pk[r / 2 + 1] = mma::h2_u32(exp2f(sc[r + 2] - m4.z) * vs, exp2f(sc[r + 3] - m4.w) * vs);
        }
        // P' row of token st: N fp16 = N/8 chunks of 16 B, MN-major swizzled (64 B / 32 B rows)
        uint8_t* prow = ps + b * L::kPBytes + st * (N * 2);
#pragma unroll
        for (int c = 0; c < N / 8; ++c) {
          const int sw = N == 32 ? (c ^ ((st >> 1) & 3)) : (c ^ ((st >> 2) & 1));
          *reinterpret_cast<uint4*>(prow + (sw << 4)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        sm100::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          sm100::mbar_arrive(&B.p_full[b]);
          if (st == 0 && i < 8) trace(tr, 40 + i);
          sm100::mbar_arrive(&B.raw_empty[s]);
        }
      }
      dead = !ok;
    }
    if (!aborted) aborted = sm100::bar_red_or(kBarSoft, 128, dead);  // every softmax warp agrees
    if (!aborted) {
      // ---- output: out[r, d] = (O^T[d, r] + C_r) / l_r
      bool ok = sm100::mbar_wait_sleep(B.stats_done, 0, abort_flag, p.status, kTimeoutAccFull, kBudgetNs);
      if (ok && n_pages > 0)
        ok = sm100::mbar_wait_sleep(&B.p_empty[(n_pages - 1) & 1], ((n_pages - 1) >> 1) & 1, abort_flag, p.status,
                              kTimeoutAccFull, kBudgetNs);
      // every softmax warp agrees before the named barrier below
      if (!sm100::bar_red_or(kBarSoft, 128, !ok)) {
        constexpr int kGroups = 64 / (N / 2);
        // per-row totals (l_r, C_r) once, into the page-maxima scratch (N x 4 floats)
        if (st < N) {
          float Lr = 0.f, Cr = 0.f;
#pragma unroll
          for (int q = 0; q < kGroups; ++q) {
            Lr += fin[q * 2 * N + st];
            Cr += fin[q * 2 * N + N + st];
          }
          const float inv = Lr > 0.f ? 1.f / Lr : 0.f;
          red[2 * st] = inv;
          red[2 * st + 1] = Cr * inv;
          if (st < nrows)
            p.part_lse[((long long)item * p.Hk + hk) * kPartRows + st] =
                Lr > 0.f ? (msm[st] + log2f(Lr)) / kLog2e : -INFINITY;
        }
        sm100::bar_sync(kBarSoft, 128);
        sm100::tc_fence_after();
        float* po = p.part_o + ((long long)item * p.Hk + hk) * kPartRows * kD;
        const float2* rc = reinterpret_cast<const float2*>(red);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t o[N];
          if (n_pages > 0) {
            if constexpr (N == 32)
              sm100::tmem_ld_32x32b_x32(tbase + lrow + kColO + h * N, o);
            else
              sm100::tmem_ld_32x32b_x16(tbase + lrow + kColO + h * N, o);
            sm100::tmem_ld_wait();
          } else {
#pragma unroll
            for (int r = 0; r < N; ++r) o[r] = 0u;
          }
          const int d = st + 128 * h;
#pragma unroll
          for (int r = 0; r < N; ++r) {
            const float2 f = rc[r];  // (1 / l_r, C_r / l_r)
            if (r < nrows) po[r * kD + d] = fmaf(__uint_as_float(o[r]), f.x, f.y);
          }
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  if (tid == 256) trace(tr, 2);  // softmax role done (outputs written)
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0) trace(tr, 3);
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, kTmemCols);
  }
}

template <int N>
int launch_tc(const AttnParams& p, cudaStream_t stream) {
  using L = TcLayout<N>;
  OSCAR_RC(ensure_smem(int2_attention_tc_kernel<N>, L::kAlloc));
  dim3 grid(p.n_work, p.Hk);
  int2_attention_tc_kernel<N><<<grid, kThreads, L::kAlloc, stream>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace
}  // namespace oscar

// Install (or, with nullptr, remove) the per-CTA timeline buffer of the tcgen05 kernel.
extern "C" int oscar_attn_tc_trace(unsigned long long* buf) {
  return (int)cudaMemcpyToSymbol(oscar::g_tc_trace, &buf, sizeof(buf));
}

// rows_per_item: the largest q_len * g - row0 of any work item (<= 32).
extern "C" int oscar_int2_attention_tc(const oscar::AttnParams* params, int rows_per_item, cudaStream_t stream) {
  using namespace oscar;
  const AttnParams& p = *params;
  if (p.n_work <= 0) return 0;
  if (p.D != kD || p.kv_mode != 0) return -330;
  if (p.page_bytes != kPageBytes) return -331;
  if (rows_per_item <= 16) return launch_tc<16>(p, stream);
  if (rows_per_item <= 32) return launch_tc<32>(p, stream);
  return -332;
}
