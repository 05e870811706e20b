// INT2 paged attention for prefill chunks on the 5th-generation tensor cores: one CTA
// per (tile of 128 query rows, KV head); rows are (token, head-in-group) pairs of one
// request, row = t * g + h.  Every row of a tile sees the whole INT2 history (keys
// before the chunk) plus the chunk's own keys up to its token (right-aligned causal).
//
// Key tiles of 128 keys:
//   history tiles  - one KV page each (positions < prefix).  The 2-bit page arrives by
//                    bulk copy; converter warps dequantise K codes (token-major) and V
//                    codes (dim-major) to fp16 values s c + z in shared memory, in the
//                    K-major 128-byte-swizzled layouts of the B operands of S = Q K^T and
//                    O += P V; staged sink/recent tokens (owner tag == block) carry their
//                    fp32 values instead.  The softmax then treats every tile alike.
//   fresh tiles    - the chunk's own (unquantised) k / v, 128 tokens at a time, loaded by
//                    TMA straight into the operand layouts (V MN-major).
// Operand chunks (16 KB: 128 keys x 64 dims of K, or 64 dims x 128 keys of V) stream
// through one FIFO ring in the order the tensor cores consume them:
//     K(0), K(1), V(0), K(2), V(1), ..., K(n-1), V(n-2), V(n-1)
// so S = Q K(i)^T overlaps the softmax of tile i-1.
//
// Roles (10 warps):
//   warps 0-3  softmax: TMEM lane = query row.  Two passes over the row's 128 scores
//              (max, then exp); running maxima move only by more than 2^8 (then O and
//              the row sums are rescaled); P' (fp16) is written into the columns of
//              its own S buffer in tensor memory - the A operand of P.V;
//   warps 4-7  converters: fill every operand chunk in FIFO order (one filler per ring,
//              so parity waits never run a phase ahead) - widened history pages, or
//              TMA boxes of fresh tiles issued by one thread;
//   warp 8     producer: bulk copies of history pages (3-slot raw ring); owns the TMEM
//              allocation;
//   warp 9     one thread issues every tcgen05.mma.
// TMEM: S0 [0,128), S1 [128,256), O [256,512) (fp32, lane = row).
//
// Every wait is bounded: an expired wait raises the CTA abort flag and records a status
// code; named-barrier groups agree on aborting with bar.red.or; bulk copies in flight
// are drained and TMEM is freed before the CTA exits.  No cluster multicast anywhere.
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
constexpr int kRows = 128;
constexpr int kPartRows = 64;  // row stride of the partials (shared with the merge)
constexpr int kThreads = 320;
constexpr int kSlots = 6;      // operand ring (16 KB chunks)
constexpr int kRaw = 3;        // raw page ring
constexpr int kPageBytes = 17408;
constexpr int kRawSlot = kPageBytes + kPage * 4;        // page + owner tags
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSlack = 8.f;
constexpr uint64_t kBudgetNs = 2000000000ull;
constexpr uint32_t kColS = 0, kColO = 256, kTmemCols = 512;
constexpr int kBarConv = 2;

struct PfLayout {
  static constexpr int kQ = 0;                                   // 4 x [128 rows][128 B]
  static constexpr int kOps = 65536;                             // kSlots x 16 KB
  static constexpr int kRawOff = kOps + kSlots * 16384;          // kRaw x kRawSlot
  static constexpr int kLim = kRawOff + kRaw * kRawSlot;         // 128 ints
  static constexpr int kSlotBlk = kLim + 512;                    // kRaw ints
  static constexpr int kTmemSlot = kSlotBlk + 16;
  static constexpr int kAbort = kTmemSlot + 16;
  static constexpr int kBars = kAbort + 16;
  // full[kSlots], empty[kSlots], raw_full[kRaw], raw_empty[kRaw], s_full[2], s_free[2], p_full[2], drain
  static constexpr int kNumBars = 2 * kSlots + 2 * kRaw + 7;
  static constexpr int kTotal = kBars + kNumBars * 8;
  static constexpr int kAlloc = kTotal + 1024;  // + base alignment
};
static_assert(PfLayout::kAlloc <= 232448, "prefill attention shared memory");

// FIFO position of the K / V chunks of tile i (n tiles): K(0), K(1), V(0), K(2), V(1), ...
OSCAR_DEVICE int use_k(int i, int c) { return i == 0 ? c : 8 * i - 4 + c; }
OSCAR_DEVICE int use_v(int i, int c, int n) { return i == n - 1 ? 8 * n - 4 + c : 8 * i + 8 + c; }

// fp16 pairs of the 64 codes of one 16-byte chunk (pool bit order: r[k] = codes 2k, 2k+1)
OSCAR_DEVICE void widen16(uint4 cw, uint32_t (&r)[32]) {
  const uint32_t w4[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t a4[4], b4[4];
    mma::codes8_to_h2(w4[q], a4);
    mma::codes8_to_h2(w4[q] >> 8, b4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      r[8 * q + e] = a4[e];
      r[8 * q + 4 + e] = b4[e];
    }
  }
}

// One 128-byte operand row (64 fp16) with the 128-byte swizzle.
OSCAR_DEVICE void store_row(uint8_t* base, int row, const uint32_t (&r)[32]) {
  uint8_t* p = base + row * 128;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<uint4*>(p + ((q ^ (row & 7)) << 4)) = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
}

// Dequantise fp16 code pairs: r[k] = r[k] * s_k + z_k (fp16x2 lanes).
OSCAR_DEVICE uint32_t hfma2_u32(uint32_t x, uint32_t s, uint32_t z) {
  __half2 v = __hfma2(*reinterpret_cast<__half2*>(&x), *reinterpret_cast<__half2*>(&s),
                      *reinterpret_cast<__half2*>(&z));
  return *reinterpret_cast<uint32_t*>(&v);
}

// Staged keys (bit set in m) of one 64-key V row take their values from the dim-major
// staging row `srow` (64 contiguous fp32).
OSCAR_DEVICE void merge_staged_v(uint32_t (&r)[32], const float* srow, uint64_t m) {
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const uint32_t b = (uint32_t)(m >> (4 * q)) & 15u;
    if (b == 0u) continue;
    const float4 v = __ldg(reinterpret_cast<const float4*>(srow) + q);
    const uint32_t lo = mma::h2_u32(v.x, v.y), hi = mma::h2_u32(v.z, v.w);
    const uint32_t k0 = ((b & 1u) ? 0u : 0x0000ffffu) | ((b & 2u) ? 0u : 0xffff0000u);
    const uint32_t k1 = ((b & 4u) ? 0u : 0x0000ffffu) | ((b & 8u) ? 0u : 0xffff0000u);
    r[2 * q] = (r[2 * q] & k0) | (lo & ~k0);
    r[2 * q + 1] = (r[2 * q + 1] & k1) | (hi & ~k1);
  }
}
// Rare path, kept out of line: K row of a staged key: 64 fp32 values of the staging arena.
__device__ __noinline__ void k_row_staged(uint8_t* base, int row, const float* sk) {
  uint32_t r[32];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(sk) + q);
    r[2 * q] = mma::h2_u32(v.x, v.y);
    r[2 * q + 1] = mma::h2_u32(v.z, v.w);
  }
  store_row(base, row, r);
}

// tiles[i] = (request, first row (multiple of 128), partial item of rows 0-63, of rows 64-127 or -1)
__global__ void __launch_bounds__(kThreads, 1)
int2_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       AttnParams p, const int4* __restrict__ tiles) {
  using L = PfLayout;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (sm100::smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* qs = smem + L::kQ;
  uint8_t* ops = smem + L::kOps;
  uint8_t* raw = smem + L::kRawOff;
  int* lim = reinterpret_cast<int*>(smem + L::kLim);
  int* slot_blk = reinterpret_cast<int*>(smem + L::kSlotBlk);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* full = bar;
  uint64_t* empty = full + kSlots;
  uint64_t* raw_full = empty + kSlots;
  uint64_t* raw_empty = raw_full + kRaw;
  uint64_t* s_full = raw_empty + kRaw;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_full + 4;
  uint64_t* drain = s_full + 6;

  const int4 tl = tiles[blockIdx.x];
  const int req = tl.x, row0 = tl.y, hk = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.Hq / p.Hk;
  const int q0 = p.q_start[req];
  const int qlen = p.q_start[req + 1] - q0;
  const int prefix = p.seq_lens[req] - qlen;
  const int* bt = p.block_tables + (long long)req * p.bt_stride;
  const int nrows = max(0, min(kRows, qlen * g - row0));
  const int t_last = nrows > 0 ? (row0 + nrows - 1) / g : -1;
  const int nh = nrows > 0 ? (prefix + kPage - 1) / kPage : 0;  // history tiles (INT2 pages)
  const int nf = nrows > 0 ? t_last / kPage + 1 : 0;             // fresh tiles (the chunk's own keys)
  const int n = nh + nf;
  const bool staging = p.stage_rows > 0;
  const float sl2 = p.scale * kLog2e;

  if (warp == 8) {
    sm100::tmem_alloc(tmem_slot, kTmemCols);
    sm100::tmem_relinquish();
  }
  if (tid == 9 * 32) {
    for (int i = 0; i < L::kNumBars; ++i) sm100::mbar_init(&bar[i], 1);
    for (int b = 0; b < 2; ++b) sm100::mbar_init(&p_full[b], 4);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (tid == 8 * 32) {
    sm100::prefetch_tmap(&tmK);
    sm100::prefetch_tmap(&tmV);
  }
  // Q tile (fp16), K-major with the 128-byte swizzle: [dim chunk of 64][row][128 B]
  for (int idx = tid; idx < kRows * 32; idx += kThreads) {
    const int r = idx >> 5, ch = idx & 31;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows) {
      const int gr = row0 + r, t = gr / g, h = gr % g;
      v = __ldg(reinterpret_cast<const uint4*>(p.q + ((long long)(q0 + t) * p.Hq + hk * g + h) * kD) + ch);
    }
    *reinterpret_cast<uint4*>(qs + (ch >> 3) * (kRows * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)) = v;
  }
  __syncthreads();
  if (tid < kRows) lim[tid] = tid < nrows ? prefix + (row0 + tid) / g : -1;
  sm100::fence_proxy_async();  // Q tile: generic writes -> tensor-core reads
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t tx = kPageBytes + (staging ? kPage * 4 : 0);
      int raw_issued = 0;
      for (int i = 0; i < nh; ++i) {  // history pages
        const int rs = i % kRaw;
        if (i >= kRaw && !sm100::mbar_wait(&raw_empty[rs], ((i / kRaw) - 1) & 1, abort_flag, p.status,
                                           kTimeoutSlotEmpty, kBudgetNs))
          break;
        const int blk = bt[i];
        slot_blk[rs] = blk;
        uint8_t* dst = raw + rs * kRawSlot;
        sm100::mbar_arrive_expect_tx(&raw_full[rs], tx);
        sm100::bulk_load(dst, p.pool + ((long long)blk * p.Hk + hk) * kPageBytes, kPageBytes, &raw_full[rs]);
        if (staging)
          sm100::bulk_load(dst + kPageBytes, p.owner + (long long)stage_row_of(p, req, i, blk) * kPage, kPage * 4,
                           &raw_full[rs]);
        raw_issued = i + 1;
      }
      if (*abort_flag) {  // copies in flight must land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        for (int i = max(0, raw_issued - kRaw); i < raw_issued; ++i)
          while (!sm100::mbar_try_wait(&raw_full[i % kRaw], (i / kRaw) & 1))
            if (globaltimer_ns() - t0 > 200000000ull) break;
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idq = sm100::idesc_f16(128, 128, false, false);
      const uint32_t idv = sm100::idesc_f16(128, 64, false, false);  // V^T chunk: K-major (dims x keys)
      const uint32_t idvf = sm100::idesc_f16(128, 64, false, true);  // fresh V: MN-major (keys x dims)
      const uint32_t qa = sm100::smem_addr(qs), oa = sm100::smem_addr(ops);
      auto wait_full = [&](int u) {
        return sm100::mbar_wait(&full[u % kSlots], (u / kSlots) & 1, abort_flag, p.status, kTimeoutTmaFull,
                                kBudgetNs);
      };
      bool ok = true;
      for (int i = 0; i <= n && ok; ++i) {
        if (i < n) {  // S(i) = Q K(i)^T
          const int b = i & 1;
          if (i >= 2 && !sm100::mbar_wait(&s_free[b], ((i >> 1) - 1) & 1, abort_flag, p.status, kTimeoutAccEmpty,
                                          kBudgetNs)) {
            ok = false;
            break;
          }
          for (int c = 0; c < 4 && ok; ++c) {
            const int u = use_k(i, c);
            if (!wait_full(u)) {
              ok = false;
              break;
            }
            sm100::tc_fence_after();
            const uint32_t kb = oa + (u % kSlots) * 16384;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sm100::smem_desc(qa + c * 16384 + kk * 32, 16, 1024, 2);
              const uint64_t bd = sm100::smem_desc(kb + kk * 32, 16, 1024, 2);
              sm100::umma_bf16(tbase + kColS + b * 128, ad, bd, idq, (c | kk) ? 1u : 0u);
            }
            sm100::umma_commit(&empty[u % kSlots]);
          }
          if (!ok) break;
          sm100::umma_commit(&s_full[b]);
        }
        if (i >= 1) {  // O += P(j) V(j)
          const int j = i - 1, b = j & 1;
          const bool fresh = j >= nh;
          if (!sm100::mbar_wait(&p_full[b], (j >> 1) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs)) {
            ok = false;
            break;
          }
          for (int c = 0; c < 4 && ok; ++c) {
            const int u = use_v(j, c, n);
            if (!wait_full(u)) {
              ok = false;
              break;
            }
            sm100::tc_fence_after();
            const uint32_t vb = oa + (u % kSlots) * 16384;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t bd = fresh ? sm100::smem_desc(vb + ks * 2048, 16384, 1024, 2)
                                        : sm100::smem_desc(vb + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, 2);
              sm100::umma_f16_tmem_a(tbase + kColO + 64 * c, tbase + kColS + b * 128 + ks * 8, bd,
                                     fresh ? idvf : idv, (j > 0 || ks > 0) ? 1u : 0u);
            }
            sm100::umma_commit(&empty[u % kSlots]);
          }
          if (!ok) break;
          sm100::umma_commit(&s_free[b]);
        }
      }
      // every MMA issued so far has completed before TMEM can be released
      sm100::umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!sm100::mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 200000000ull) break;
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ converters: every operand chunk
    const int ct = tid - 128;
    bool ok = true;
    int last_tma = -1;  // last use filled by TMA (ct == 0)
    for (int i = 0; i <= n; ++i) {
      for (int part = 0; part < 2; ++part) {
        // part 0: K(i); part 1: V(i - 1)
        const int ti = part == 0 ? i : i - 1;
        if (ti < 0 || (part == 0 && i >= n)) continue;
        const bool hist = ti < nh;
        const int rs = ti % kRaw;
        const uint8_t* pg = raw + rs * kRawSlot;
        const int* own = reinterpret_cast<const int*>(pg + kPageBytes);
        if (hist && part == 0 && ok)
          ok = sm100::mbar_wait(&raw_full[rs], (ti / kRaw) & 1, abort_flag, p.status, kTimeoutTmaFull, kBudgetNs);
        ok = __all_sync(0xffffffffu, ok);
        const int blk = hist ? slot_blk[rs] : 0;
        const int nvalid = hist ? min(kPage, prefix - kPage * ti) : 0;
        // staged keys of this page, as 128-bit masks every warp computes for itself
        uint32_t smk[4] = {0u, 0u, 0u, 0u};
        if (hist && staging) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int tj = 32 * q + lane;
            smk[q] = __ballot_sync(0xffffffffu, ok && tj < nvalid && own[tj] == blk);
          }
        }
        // dequantisation constants: K - this thread's key; V - lane l holds the fp16
        // (scale, zero) pairs of keys 64 hf + 2 l, + 1 (broadcast by shuffles); keys past
        // the history get zero scale and zero so stale meta cannot leak in
        const __half* meta = reinterpret_cast<const __half*>(pg + 2 * kPage * 64);
        uint32_t ks2 = 0u, kz2 = 0u, vsp = 0u, vzp = 0u;
        if (hist && ok) {
          if (part == 0) {
            const int j = ct;
            if (j < nvalid) {
              const __half ks = meta[j], kz = meta[kPage + j];
              const __half2 s2 = __halves2half2(ks, ks), z2 = __halves2half2(kz, kz);
              ks2 = *reinterpret_cast<const uint32_t*>(&s2);
              kz2 = *reinterpret_cast<const uint32_t*>(&z2);
            }
          } else {
            const int kb = 64 * (ct >> 6) + 2 * lane;
            vsp = *reinterpret_cast<const uint32_t*>(meta + 2 * kPage + kb);
            vzp = *reinterpret_cast<const uint32_t*>(meta + 3 * kPage + kb);
            const uint32_t keep = (kb < nvalid ? 0x0000ffffu : 0u) | (kb + 1 < nvalid ? 0xffff0000u : 0u);
            vsp &= keep;
            vzp &= keep;
          }
        }
        for (int c = 0; c < 4; ++c) {
          const int u = part == 0 ? use_k(ti, c) : use_v(ti, c, n);
          const int s = u % kSlots;
          if (ok && u >= kSlots)
            ok = sm100::mbar_wait(&empty[s], ((u / kSlots) - 1) & 1, abort_flag, p.status, kTimeoutAccEmpty,
                                  kBudgetNs);
          ok = __all_sync(0xffffffffu, ok);  // warp-uniform before the shuffles below
          uint8_t* dst = ops + s * 16384;
          if (ok && !hist) {
            // fresh tile: one TMA box (128 tokens x 64 dims) of k or v
            if (ct == 0) {
              sm100::mbar_arrive_expect_tx(&full[s], 16384);
              sm100::tma_load_2d(dst, part == 0 ? &tmK : &tmV, &full[s], hk * kD + 64 * c,
                                 q0 + kPage * (ti - nh));
              last_tma = u;
            }
          } else if (ok) {
            if (part == 0) {
              // K rows: key ct, dims 64c .. 64c + 63
              const int j = ct;
              if ((smk[j >> 5] >> (j & 31)) & 1u) {
                k_row_staged(dst, j,
                             p.stage_k + ((long long)(stage_row_of(p, req, ti, blk) * kPage + j) * p.Hk + hk) * kD +
                                 64 * c);
              } else {
                const uint4 cw = *reinterpret_cast<const uint4*>(pg + j * 64 + ((c ^ ((j >> 1) & 3)) << 4));
                uint32_t r[32];
                widen16(cw, r);
#pragma unroll
                for (int k = 0; k < 32; ++k) r[k] = hfma2_u32(r[k], ks2, kz2);
                store_row(dst, j, r);
              }
            } else {
              // V^T rows: dim 64c + dl, keys 64 hf .. 64 hf + 63
              const int dl = ct & 63, hf = ct >> 6, d = 64 * c + dl;
              const uint4 cw = *reinterpret_cast<const uint4*>(pg + kPage * 64 + d * 32 + hf * 16);
              const uint64_t m = ((uint64_t)smk[2 * hf + 1] << 32) | smk[2 * hf];
              uint32_t r[32];
              widen16(cw, r);
#pragma unroll
              for (int k = 0; k < 32; ++k)
                r[k] = hfma2_u32(r[k], __shfl_sync(0xffffffffu, vsp, k), __shfl_sync(0xffffffffu, vzp, k));
              if (m != 0ull)  // warp-uniform: staged keys carry their own values
                merge_staged_v(r, p.stage_v + ((long long)stage_row_of(p, req, ti, blk) * p.Hk + hk) * kD * kPage +
                                      (long long)d * kPage + hf * 64,
                               m);
              store_row(dst + hf * 8192, dl, r);
            }
            sm100::fence_proxy_async();  // generic writes -> tensor-core reads
          }
          if (sm100::bar_red_or(kBarConv, 128, !ok)) {
            ok = false;
            break;
          }
          if (ct == 0 && hist) sm100::mbar_arrive(&full[s]);
        }
        if (!ok) break;
        if (part == 1 && hist && ct == 0) sm100::mbar_arrive(&raw_empty[rs]);
      }
      if (!ok) break;
    }
    if (ct == 0 && *abort_flag && last_tma >= 0) {  // TMA boxes in flight must land before the CTA exits
      const uint64_t t0 = globaltimer_ns();
      for (int u = max(0, last_tma - kSlots + 1); u <= last_tma; ++u)
        while (!sm100::mbar_try_wait(&full[u % kSlots], (u / kSlots) & 1))
          if (globaltimer_ns() - t0 > 200000000ull) break;
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 0-3)
    const int r = tid;  // TMEM lane = query row
    const uint32_t lrow = (uint32_t)(warp * 32) << 16;
    const int my_lim = lim[r];
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
      const int b = i & 1;
      const bool hist = i < nh;
      ok = sm100::mbar_wait(&s_full[b], (i >> 1) & 1, abort_flag, p.status, kTimeoutAccFull, kBudgetNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      sm100::tc_fence_after();
      // visible keys of this tile for this row: j < jmax
      const int jmax = hist ? min(kPage, prefix - kPage * i) : max(0, min(kPage, my_lim - prefix - kPage * (i - nh) + 1));
      const uint32_t sb = tbase + lrow + kColS + b * 128;
      // ---- pass 1: row maximum of the tile
      float pm = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t raw32[32];
        sm100::tmem_ld_32x32b_x32(sb + 32 * c, raw32);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = 32 * c + e;
          pm = j < jmax ? fmaxf(pm, __uint_as_float(raw32[e])) : pm;
        }
      }
      pm *= sl2;  // log2 units
      // ---- running maximum: moves only when exceeded by more than 2^kSlack
      float alpha = 1.f;
      if (pm > m + kSlack) {
        alpha = m == -INFINITY ? 0.f : exp2f(m - pm);
        m = pm;
        l *= alpha;
      }
      if (__any_sync(0xffffffffu, alpha != 1.f) && i > 0) {
        // O holds tiles < i: rescale this warp's rows once P.V(i-1) is done
        ok = sm100::mbar_wait(&s_free[(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag, p.status, kTimeoutAccFull,
                              kBudgetNs);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        sm100::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[32];
          sm100::tmem_ld_32x32b_x32(tbase + lrow + kColO + 32 * c, o);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          sm100::tmem_st_32x32b_x32(tbase + lrow + kColO + 32 * c, o);
        }
        sm100::tmem_st_wait();
      }
      // ---- pass 2: P' = p s_v (fp16) into the first 64 columns of this S buffer
      const float mref = m == -INFINITY ? 0.f : m;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t raw32[32], pk[16];
        sm100::tmem_ld_32x32b_x32(sb + 32 * c, raw32);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int j = 32 * c + e;
          const float p0 = j < jmax ? exp2f(fmaf(__uint_as_float(raw32[e]), sl2, -mref)) : 0.f;
          const float p1 = j + 1 < jmax ? exp2f(fmaf(__uint_as_float(raw32[e + 1]), sl2, -mref)) : 0.f;
          const __half2 h = __floats2half2_rn(p0, p1);
          const float2 hf = __half22float2(h);
          l += hf.x + hf.y;  // the row sum of exactly the P the tensor cores read
          pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&h);
        }
        sm100::tmem_st_32x32b_x16(sb + 16 * c, pk);
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&p_full[b]);
    }
    // ---- output: out[r, d] = O[r, d] / l_r  into the 64-row partials
    if (ok && n > 0)
      ok = sm100::mbar_wait(&s_free[(n - 1) & 1], ((n - 1) >> 1) & 1, abort_flag, p.status, kTimeoutAccFull,
                            kBudgetNs);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      sm100::tc_fence_after();
      const int item = r < 64 ? tl.z : tl.w;
      const bool write = r < nrows && item >= 0;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float* po = p.part_o + (((long long)(write ? item : 0) * p.Hk + hk) * kPartRows + (r & 63)) * kD;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t o[32];
        if (n > 0) {
          sm100::tmem_ld_32x32b_x32(tbase + lrow + kColO + 32 * c, o);
          sm100::tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (write) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(po + 32 * c + e) =
                make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                            __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
        }
      }
      if (write)
        p.part_lse[((long long)item * p.Hk + hk) * kPartRows + (r & 63)] =
            l > 0.f ? (m + log2f(l)) / kLog2e : -INFINITY;
    }
  }

  // ---------------------------------------------------------------- teardown
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tbase, kTmemCols);
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

// fresh k / v [rows = tokens][cols = Hk * D] fp16 viewed 2-D; boxes of 128 rows x 64 cols
// with the 128-byte swizzle (rows past the end read as zeros).
int fresh_map(CUtensorMap* map, const void* base, long long rows, long long cols) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::pair<long long, CUtensorMap>> cache;
  const long long key = rows * 1000003 + cols;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(base);
    if (it != cache.end() && it->second.first == key) {
      *map = it->second.second;
      return 0;
    }
  }
  EncodeFn enc = encode_fn();
  if (!enc) return -360;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -361;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 256) cache.clear();
  cache[base] = {key, *map};
  return 0;
}

}  // namespace
}  // namespace oscar

// INT2 prefill tiles: `tiles` [n_tiles] int4 (request, first row, item of rows 0-63, item of
// rows 64-127 or -1) on the device; fresh_rows = token rows of k_fresh / v_fresh.
extern "C" int oscar_int2_prefill_tc(const oscar::AttnParams* params, const void* tiles, int n_tiles,
                                     long long fresh_rows, cudaStream_t stream) {
  using namespace oscar;
  const AttnParams& p = *params;
  if (n_tiles <= 0) return 0;
  if (p.D != kD || p.kv_mode != 0 || !p.pool || p.page_bytes != kPageBytes) return -362;
  if ((reinterpret_cast<uintptr_t>(p.k_fresh) & 15) || (reinterpret_cast<uintptr_t>(p.v_fresh) & 15)) return -363;
  CUtensorMap tk, tv;
  int rc = fresh_map(&tk, p.k_fresh, fresh_rows, (long long)p.Hk * kD);
  if (rc) return rc;
  rc = fresh_map(&tv, p.v_fresh, fresh_rows, (long long)p.Hk * kD);
  if (rc) return rc;
  OSCAR_RC(ensure_smem(int2_prefill_tc_kernel, PfLayout::kAlloc));
  dim3 grid(n_tiles, p.Hk);
  int2_prefill_tc_kernel<<<grid, kThreads, PfLayout::kAlloc, stream>>>(tk, tv, p,
                                                                         reinterpret_cast<const int4*>(tiles));
  return (int)cudaGetLastError();
}
