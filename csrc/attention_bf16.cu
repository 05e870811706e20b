// BF16-KV paged attention on the tensor cores (tcgen05 + TMEM), for work items of at
// most 32 query rows.  It serves the MTP draft layer, whose cache stays BF16
// (`[blocks, 128, Hk, D]`, the shadow pool), and BF16-KV runs of the full layers.
//
// One CTA per (work item, KV head), 8 warps:
//   warp 0     TMA producer: each page-head arrives as eight [128 tokens x 64 dims]
//              boxes with the 128-byte swizzle - K boxes are the K-major A operand of
//              S^T = K Q^T, V boxes the MN-major A operand of O^T += V^T P^T - into a
//              ring of 32 KB pair slots (K0K1, K2K3, V0V1, V2V3 per page);
//   warp 1     one thread issues every tcgen05.mma (A and B from shared memory);
//   warps 2-3  row statistics: l_r = sum_j p_jr from the bf16 P tile the tensor cores read;
//   warps 4-7  softmax: TMEM lane t = token t; running maxima move only when a score
//              exceeds them by more than 2^8 (then O^T is rescaled in TMEM).
// All tokens, the current chunk's included, are read from the cache: the step's store
// writes them before attention runs.  Bounded waits everywhere; no cluster multicast.
#include <cuda.h>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "mma.cuh"
#include "params.h"
#include "sm100.cuh"

namespace oscar {
namespace {

constexpr int kD = 256;
constexpr int kPage = 128;
constexpr int kPartRows = 64;
constexpr int kPairs = 5;               // ring of 32 KB pair slots
constexpr int kPairBytes = 2 * 16384;   // two [128 x 64] bf16 boxes
constexpr int kThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSlack = 8.f;
constexpr uint64_t kBudgetNs = 2000000000ull;
constexpr int kBarSoft = 1, kBarStats = 3;

template <int N>
struct BfLayout {
  static constexpr int kQOff = kPairs * kPairBytes;  // 163,840: 1024-aligned
  static constexpr int kPOff = kQOff + N * 512;      // Q: 4 chunks x N rows x 128 B (bf16)
  static constexpr int kPBytes = kPage * N * 2;      // one P buffer: 128 tokens x N bf16
  static constexpr int kMisc = kPOff + 2 * kPBytes;
  static constexpr int kLim = kMisc;                 // N ints
  static constexpr int kMsm = kLim + N * 4;          // N floats
  static constexpr int kRed = kMsm + N * 4;          // N x 4 floats
  static constexpr int kAlpha = kRed + N * 16;       // 2 x N floats
  static constexpr int kFin = kAlpha + 2 * N * 4;    // groups x N floats
  static constexpr int kFlags = kFin + 512;          // upd[2], resc
  static constexpr int kTmemSlot = kFlags + 16;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kBars = (kAbort + 4 + 7) / 8 * 8;
  // full[kPairs], empty[kPairs], s_full[2], s_empty[2], p_full[2], p_empty[2], mma_done, stats_done
  static constexpr int kNumBars = 2 * kPairs + 8 + 2;
  static constexpr int kTotal = kBars + kNumBars * 8 + 1024;  // + base alignment
};

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
__global__ void __launch_bounds__(kThreads, 1)
bf16_attention_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         AttnParams p) {
  using L = BfLayout<N>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (sm100::smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  uint8_t* qs = smem + L::kQOff;
  uint8_t* ps = smem + L::kPOff;
  int* lim = reinterpret_cast<int*>(smem + L::kLim);
  float* msm = reinterpret_cast<float*>(smem + L::kMsm);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* alpha = reinterpret_cast<float*>(smem + L::kAlpha);
  float* fin = reinterpret_cast<float*>(smem + L::kFin);
  volatile int* upd = reinterpret_cast<volatile int*>(smem + L::kFlags);
  volatile int* resc_flag = reinterpret_cast<volatile int*>(smem + L::kFlags + 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* full = bar;
  uint64_t* empty = bar + kPairs;
  uint64_t* s_full = bar + 2 * kPairs;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_full + 4;
  uint64_t* p_empty = s_full + 6;
  uint64_t* mma_done = s_full + 8;
  uint64_t* stats_done = s_full + 9;

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
  const int p_first = kv_begin / kPage;
  const int n_pages = kv_stop > kv_begin ? (kv_stop - 1) / kPage - p_first + 1 : 0;
  constexpr uint32_t kCols = 4 * N < 32 ? 32 : 4 * N;  // S (2 x N) + O (2 x N)

  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, kCols);
    sm100::tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < L::kNumBars; ++i) sm100::mbar_init(&bar[i], 1);
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&s_empty[b], 4);
      sm100::mbar_init(&p_full[b], 4);
      sm100::mbar_init(&p_empty[b], 3);  // P.V commit + 2 stats warps
    }
    sm100::mbar_init(stats_done, 2);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    sm100::prefetch_tmap(&tmK);
    sm100::prefetch_tmap(&tmV);
  }
  // Q tile (bf16), K-major with the 128-byte swizzle: [dim chunk][row][128 B]
  for (int idx = tid; idx < N * 32; idx += kThreads) {
    const int r = idx >> 5, ch = idx & 31;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows) {
      const int gr = row0 + r, t = gr / g, h = gr % g;
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(p.q + ((long long)(q0 + t) * p.Hq + hk * g + h) * kD) + ch);
      const __half2* hx = reinterpret_cast<const __half2*>(&x);
      uint32_t* o = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(hx[e]);
        o[e] = pack_bf16x2(f.x, f.y);
      }
    }
    *reinterpret_cast<uint4*>(qs + (ch >> 3) * (N * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)) = v;
  }
  if (tid < N) {
    lim[tid] = tid < nrows ? prefix + (row0 + tid) / g : -1;
    msm[tid] = -INFINITY;
  }
  sm100::fence_proxy_async();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t kColS = 0, kColO = 2 * N;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < n_pages && ok; ++i) {
        const int blk = bt[p_first + i];
        for (int q = 0; q < 4; ++q) {
          const int u = 4 * i + q, s = u % kPairs;
          if (u >= kPairs && !sm100::mbar_wait(&empty[s], ((u / kPairs) - 1) & 1, abort_flag, p.status,
                                               kTimeoutSlotEmpty, kBudgetNs)) {
            ok = false;
            break;
          }
          uint8_t* dst = ring + s * kPairBytes;
          sm100::mbar_arrive_expect_tx(&full[s], kPairBytes);
          const CUtensorMap* tm = q < 2 ? &tmK : &tmV;
          const int c0 = 2 * (q & 1);  // first 64-dim chunk of the pair
          sm100::tma_load_2d(dst, tm, &full[s], hk * kD + 64 * c0, blk * kPage);
          sm100::tma_load_2d(dst + 16384, tm, &full[s], hk * kD + 64 * (c0 + 1), blk * kPage);
          issued = u + 1;
        }
      }
      if (*abort_flag) {
        const uint64_t t0 = globaltimer_ns();
        for (int u = max(0, issued - kPairs); u < issued; ++u)
          while (!sm100::mbar_try_wait(&full[u % kPairs], (u / kPairs) & 1))
            if (globaltimer_ns() - t0 > 200000000ull) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idq = sm100::idesc_bf16(128, N, false, false);
      const uint32_t idp = sm100::idesc_bf16(128, N, true, true);
      const uint32_t qa = sm100::smem_addr(qs), pa = sm100::smem_addr(ps), ra = sm100::smem_addr(ring);
      constexpr uint32_t kPLayout = N == 32 ? 4u : 6u;
      constexpr uint32_t kPAtom = 8 * N * 2;
      auto wait_full = [&](int u) {
        return sm100::mbar_wait(&full[u % kPairs], (u / kPairs) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs);
      };
      auto pv = [&](int j) -> bool {
        if (!wait_full(4 * j + 2) || !wait_full(4 * j + 3)) return false;
        if (!sm100::mbar_wait(&p_full[j & 1], (j >> 1) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs))
          return false;
        sm100::tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t vbase = ra + ((4 * j + 2 + h) % kPairs) * kPairBytes;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            // V^T half h: MN-major, 64-dim chunks 16 KB apart (LBO), 8-token groups 1 KB apart
            const uint64_t ad = sm100::smem_desc(vbase + ks * 2048, 16384, 1024, 2);
            const uint64_t bd = sm100::smem_desc(pa + (j & 1) * L::kPBytes + ks * 2 * kPAtom, 16, kPAtom, kPLayout);
            sm100::umma_bf16(tbase + kColO + h * N, ad, bd, idp, (j > 0 || ks > 0) ? 1u : 0u);
          }
        }
        sm100::umma_commit(&empty[(4 * j + 2) % kPairs]);
        sm100::umma_commit(&empty[(4 * j + 3) % kPairs]);
        sm100::umma_commit(&p_empty[j & 1]);
        return true;
      };
      bool ok = true;
      for (int i = 0; i < n_pages && ok; ++i) {
        if (!wait_full(4 * i) || !wait_full(4 * i + 1)) {
          ok = false;
          break;
        }
        if (i >= 2 && !sm100::mbar_wait(&s_empty[i & 1], ((i >> 1) - 1) & 1, abort_flag, p.status,
                                        kTimeoutAccEmpty, kBudgetNs)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const int c = kk >> 2;
          const uint32_t kbase = ra + ((4 * i + (c >> 1)) % kPairs) * kPairBytes + (c & 1) * 16384;
          const uint64_t ad = sm100::smem_desc(kbase + (kk & 3) * 32, 16, 1024, 2);
          const uint64_t qd = sm100::smem_desc(qa + c * (N * 128) + (kk & 3) * 32, 16, 1024, 2);
          sm100::umma_bf16(tbase + kColS + (i & 1) * N, ad, qd, idq, kk > 0 ? 1u : 0u);
        }
        sm100::umma_commit(&s_full[i & 1]);
        sm100::umma_commit(&empty[(4 * i) % kPairs]);
        sm100::umma_commit(&empty[(4 * i + 1) % kPairs]);
        if (i >= 1) ok = pv(i - 1);
      }
      if (ok && n_pages > 0) pv(n_pages - 1);
      sm100::umma_commit(mma_done);
      const uint64_t t0 = globaltimer_ns();
      while (!sm100::mbar_try_wait(mma_done, 0))
        if (globaltimer_ns() - t0 > 200000000ull) break;
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ row sums from the P tile
    const int tt = tid - 64;
    constexpr int kPr = N / 2, kGroups = 64 / kPr, kTok = kPage / kGroups;
    const int rp = tt % kPr, grp = tt / kPr;
    float l0 = 0.f, l1 = 0.f;
    bool aborted = false;
    for (int i = 0; i < n_pages; ++i) {
      const int b = i & 1;
      const bool ok = sm100::mbar_wait(&p_full[b], (i >> 1) & 1, abort_flag, p.status, kTimeoutAccFull, kBudgetNs);
      if (sm100::bar_red_or(kBarStats, 64, !ok)) {
        aborted = true;
        break;
      }
      if (upd[b]) {
        l0 *= alpha[b * N + 2 * rp];
        l1 *= alpha[b * N + 2 * rp + 1];
      }
      const uint8_t* pt = ps + b * L::kPBytes;
#pragma unroll 4
      for (int k = 0; k < kTok; ++k) {
        const int j = grp * kTok + k;
        const int c = (2 * rp) >> 3;
        const int sw = N == 32 ? (c ^ ((j >> 1) & 3)) : (c ^ ((j >> 2) & 1));
        const uint32_t hv = *reinterpret_cast<const uint32_t*>(pt + j * (N * 2) + (sw << 4) + ((2 * rp) & 7) * 2);
        const float2 pf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hv));
        l0 += pf.x;
        l1 += pf.y;
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&p_empty[b]);
    }
    if (!aborted) {
      fin[grp * N + 2 * rp] = l0;
      fin[grp * N + 2 * rp + 1] = l1;
    }
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(stats_done);
  } else {
    // ------------------------------------------------------------ softmax (warps 4-7)
    const int st = tid - 128;
    const int swarp = st >> 5;
    const uint32_t lrow = (uint32_t)(st & ~31) << 16;
    const float sl2 = p.scale * kLog2e;
    // per-row constants in registers (lane r holds row r), broadcast by shuffles
    const int lim_l = lim[lane % N];
    float m_l = msm[lane % N];
    bool dead = false, aborted = false;
    for (int i = 0; i < n_pages; ++i) {
      const int b = i & 1;
      bool ok = !dead && sm100::mbar_wait(&s_full[b], (i >> 1) & 1, abort_flag, p.status, kTimeoutAccFull,
                                          kBudgetNs);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform before the shuffles below
      float sc[N];
      bool need = false;
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
        if (lane == 0) sm100::mbar_arrive(&s_empty[b]);
        const int pos = (p_first + i) * kPage + st;
        const bool in = pos >= kv_begin && pos < kv_stop;
        const bool hist = pos < prefix;
#pragma unroll
        for (int r = 0; r < N; ++r) {
          // every lane takes part in both shuffles (no short-circuit around them)
          const int lv = __shfl_sync(0xffffffffu, lim_l, r);
          const float mv = __shfl_sync(0xffffffffu, m_l, r);
          const bool vis = in && (hist || pos <= lv);
          sc[r] = vis ? __uint_as_float(raw[r]) * sl2 : -INFINITY;
          need |= sc[r] > mv + kSlack;
        }
      }
      if (ok && i >= 2)
        ok = sm100::mbar_wait(&p_empty[b], ((i >> 1) - 1) & 1, abort_flag, p.status, kTimeoutAccEmpty, kBudgetNs);
      if (sm100::bar_red_or(kBarSoft, 128, !ok)) {
        aborted = true;
        break;
      }
      const bool upd_now = sm100::bar_red_or(kBarSoft, 128, need);
      if (upd_now) {
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
        m_l = msm[lane % N];
        if (*resc_flag && i > 0) {
          const bool ok2 = sm100::mbar_wait(&p_empty[(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag, p.status,
                                            kTimeoutAccFull, kBudgetNs);
          if (ok2) {
            sm100::tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t o[N];
              if constexpr (N == 32)
                sm100::tmem_ld_32x32b_x32(tbase + lrow + kColO + h * N, o);
              else
                sm100::tmem_ld_32x32b_x16(tbase + lrow + kColO + h * N, o);
              sm100::tmem_ld_wait();
#pragma unroll
              for (int r = 0; r < N; ++r) o[r] = __float_as_uint(__uint_as_float(o[r]) * alpha[b * N + r]);
              if constexpr (N == 32)
                sm100::tmem_st_32x32b_x32(tbase + lrow + kColO + h * N, o);
              else
                sm100::tmem_st_32x32b_x16(tbase + lrow + kColO + h * N, o);
            }
            sm100::tmem_st_wait();
            sm100::tc_fence_before();
          }
          ok = ok2;
        }
      }
      if (st == 0) upd[b] = upd_now ? 1 : 0;
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        uint32_t pk[N / 2];
        const float mref_l = m_l == -INFINITY ? 0.f : m_l;
#pragma unroll
        for (int r = 0; r < N; r += 2) {
          const float p0 = exp2f(sc[r] - __shfl_sync(0xffffffffu, mref_l, r));
          const float p1 = exp2f(sc[r + 1] - __shfl_sync(0xffffffffu, mref_l, r + 1));
          pk[r / 2] = pack_bf16x2(p0, p1);
        }
        uint8_t* prow = ps + b * L::kPBytes + st * (N * 2);
#pragma unroll
        for (int c = 0; c < N / 8; ++c) {
          const int sw = N == 32 ? (c ^ ((st >> 1) & 3)) : (c ^ ((st >> 2) & 1));
          *reinterpret_cast<uint4*>(prow + (sw << 4)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        sm100::fence_proxy_async();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&p_full[b]);
      }
      dead = !ok;
    }
    if (!aborted) aborted = sm100::bar_red_or(kBarSoft, 128, dead);
    if (!aborted) {
      bool ok = sm100::mbar_wait(stats_done, 0, abort_flag, p.status, kTimeoutAccFull, kBudgetNs);
      if (ok && n_pages > 0)
        ok = sm100::mbar_wait(&p_empty[(n_pages - 1) & 1], ((n_pages - 1) >> 1) & 1, abort_flag, p.status,
                              kTimeoutAccFull, kBudgetNs);
      if (ok) {
        constexpr int kGroups = 64 / (N / 2);
        sm100::tc_fence_after();
        float* po = p.part_o + ((long long)item * p.Hk + hk) * kPartRows * kD;
#pragma unroll
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
            if (r >= nrows) break;
            float Lr = 0.f;
#pragma unroll
            for (int q = 0; q < kGroups; ++q) Lr += fin[q * N + r];
            po[r * kD + d] = Lr > 0.f ? __uint_as_float(o[r]) / Lr : 0.f;
          }
        }
        if (st < nrows) {
          float Lr = 0.f;
#pragma unroll
          for (int q = 0; q < kGroups; ++q) Lr += fin[q * N + st];
          p.part_lse[((long long)item * p.Hk + hk) * kPartRows + st] =
              Lr > 0.f ? (msm[st] + log2f(Lr)) / kLog2e : -INFINITY;
        }
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, kCols);
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// [rows = blocks * 128][cols = Hk * D] bf16 cache viewed 2-D; boxes of 128 rows x 64 cols.
int cache_map(CUtensorMap* map, const void* base, long long rows, long long cols) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::pair<long long, CUtensorMap>> cache;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(base);
    if (it != cache.end() && it->second.first == rows * 1000003 + cols) {
      *map = it->second.second;
      return 0;
    }
  }
  EncodeFn enc = encode_fn();
  if (!enc) return -340;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -341;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 256) cache.clear();
  cache[base] = {rows * 1000003 + cols, *map};
  return 0;
}

template <int N>
int launch_bf16(const CUtensorMap& tk, const CUtensorMap& tv, const AttnParams& p, cudaStream_t stream) {
  using L = BfLayout<N>;
  OSCAR_RC(ensure_smem(bf16_attention_tc_kernel<N>, L::kTotal));
  dim3 grid(p.n_work, p.Hk);
  bf16_attention_tc_kernel<N><<<grid, kThreads, L::kTotal, stream>>>(tk, tv, p);
  return (int)cudaGetLastError();
}

}  // namespace
}  // namespace oscar

// BF16 pages (kv_mode 1); num_blocks = pool blocks of kc / vc; rows_per_item <= 32.
extern "C" int oscar_bf16_attention_tc(const oscar::AttnParams* params, long long num_blocks, int rows_per_item,
                                       cudaStream_t stream) {
  using namespace oscar;
  const AttnParams& p = *params;
  if (p.n_work <= 0) return 0;
  if (p.D != kD || p.kv_mode != 1 || !p.kc || !p.vc) return -342;
  if ((reinterpret_cast<uintptr_t>(p.kc) & 15) || (reinterpret_cast<uintptr_t>(p.vc) & 15)) return -343;
  CUtensorMap tk, tv;
  int rc = cache_map(&tk, p.kc, num_blocks * kPage, (long long)p.Hk * kD);
  if (rc) return rc;
  rc = cache_map(&tv, p.vc, num_blocks * kPage, (long long)p.Hk * kD);
  if (rc) return rc;
  if (rows_per_item <= 16) return launch_bf16<16>(tk, tv, p, stream);
  if (rows_per_item <= 32) return launch_bf16<32>(tk, tv, p, stream);
  return -344;
}
