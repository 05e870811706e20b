// W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
//   D[m, n] = sum_k A[m, k] * B[n, k]            (int8 x int8 -> int32 in TMEM)
//   out     = D * scale_a[m] * scale_b[n]        (bf16 store, fp32 store or fp32 atomic add)
//
// Both operands are K-major int8 and are brought into shared memory by TMA with
// the 128-byte swizzle (one 128-byte K slab per tile row).  The CTA is warp
// specialised: warp 0 issues TMA loads, warp 1 allocates TMEM and one elected
// thread issues tcgen05.mma, warps 2..5 drain the accumulator from TMEM with
// tcgen05.ld and run the dequantising epilogue.  The kernel is persistent
// (grid = number of SMs) and double-buffers the TMEM accumulator so that the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// A linear layer y = x W^T calls it either with (A=x, B=W) for large token
// counts or "swapped" with (A=W, B=x) for decode-sized batches, where the token
// count becomes the MMA N dimension; split-K (fp32 atomics into the output)
// keeps all SMs streaming weights when there are few output tiles.  The fp32
// atomic mode is also how row-parallel projections add straight into the fp32
// residual stream.
#include <cuda.h>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include "sm100.cuh"
#include "params.h"

namespace oscar {


namespace {

constexpr int BM = 128;
constexpr int BK = 128;           // bytes of K per stage (one 128 B swizzle row)
constexpr int UMMA_K = 32;        // K per tcgen05.mma kind::i8
constexpr int kThreads = 192;
constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196 * 1024) / STAGE_BYTES > 8 ? 8 : (196 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Reduce-scatter epilogue (mode 5): the fp32 value(s) of token `tok`, output
// column(s) `col..` go to the rank owning that token, stored over NVLink into this
// rank's slot of the owner's receive buffer (every value is written once; the owner
// adds the slots of all ranks in a fixed order).
OSCAR_DEVICE float* owner_dst(const GemmEpi& ep, int tok, int col) {
  const int owner = tok / ep.rows_per_rank;
  return ep.peer_out[owner] + ep.rank * ep.slot_stride + (long long)(tok - owner * ep.rows_per_rank) * ep.ldo + col;
}
OSCAR_DEVICE void red_to_owner(const GemmEpi& ep, int tok, int col, float4 v) {
  *reinterpret_cast<float4*>(owner_dst(ep, tok, col)) = v;
}
OSCAR_DEVICE void red_to_owner1(const GemmEpi& ep, int tok, int col, float v) { *owner_dst(ep, tok, col) = v; }

// One output value of a finished (fully reduced) element; used by the cluster
// reduction for tails that do not fill a 4-wide vector.
OSCAR_DEVICE void store_one(const GemmEpi& ep, int m, int n, float v) {
  const long long idx = ep.trans ? (long long)n * ep.ldo + m : (long long)m * ep.ldo + n;
  switch (ep.mode) {
    case 0:
    case 4: reinterpret_cast<__nv_bfloat16*>(ep.out)[idx] = __float2bfloat16(v); break;
    case 1: atomicAdd(reinterpret_cast<float*>(ep.out) + idx, v); break;
    case 2: reinterpret_cast<float*>(ep.out)[idx] = v; break;
    case 3:
      asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(reinterpret_cast<float*>(ep.out) + idx),
                   "f"(v)
                   : "memory");
      break;
    case 5: red_to_owner1(ep, ep.trans ? n : m, ep.trans ? m : n, v); break;
  }
}
// Four consecutive output values at out index `idx` (16-byte aligned in fp32 terms).
OSCAR_DEVICE void store_four(const GemmEpi& ep, long long idx, int tok, int col, float4 v) {
  switch (ep.mode) {
    case 0:
    case 4:
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(ep.out) + idx) =
          make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      break;
    case 1:
      asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                       reinterpret_cast<float*>(ep.out) + idx),
                   "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                   : "memory");
      break;
    case 2: *reinterpret_cast<float4*>(reinterpret_cast<float*>(ep.out) + idx) = v; break;
    case 3:
      asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                       reinterpret_cast<float*>(ep.out) + idx),
                   "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                   : "memory");
      break;
    case 5: red_to_owner(ep, tok, col, v); break;
  }
}

// Split-K through the cluster: CTA `me` of `S` (any S <= 8) sums its share of the
// tile's rows - whole groups of 4 rows, [4*floor(32*me/S), 4*floor(32*(me+1)/S)) - of
// the S partial int32 tiles that the CTAs staged in their shared memory (`red`,
// [BN][BM+4] for the swapped layout, [BM][BN+4] otherwise), scales them and writes the
// result.
template <int BN>
OSCAR_DEVICE void cluster_reduce_tile(const GemmEpi& ep, const int32_t* red, int m0, int n0, int M, int N, int e) {
  constexpr int RS = BM + 4, CS = BN + 4;
  const int S = ep.cluster_k;
  const uint32_t me = sm100::cluster_ctarank();
  const int r0 = 4 * ((BM / 4) * (int)me / S), R = 4 * ((BM / 4) * ((int)me + 1) / S) - r0;
  const uint32_t base = smem_u32(red);
  const bool vec_ok = (ep.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(ep.out) & 15) == 0;
  if (ep.trans) {
    // output (m, n) at out[n * ldo + m]: vectors of 4 consecutive m of one column n
    const int per_col = R / 4;
    for (int v = e; v < per_col * BN; v += 128) {
      const int col = v / per_col, m4 = r0 + 4 * (v % per_col);
      const int n = n0 + col, m = m0 + m4;
      if (n >= N || m >= M) continue;
      const uint32_t a = base + (uint32_t)(col * RS + m4) * 4u;
      int4 acc = sm100::ld_dsmem_v4(sm100::mapa(a, 0));
      for (int q = 1; q < S; ++q) {
        const int4 x = sm100::ld_dsmem_v4(sm100::mapa(a, q));
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
      const float sb = __ldg(ep.scale_b + n);
      if (m + 3 < M && (vec_ok || ep.mode == 5) && (reinterpret_cast<uintptr_t>(ep.scale_a + m) & 15) == 0) {
        const float4 sa = __ldg(reinterpret_cast<const float4*>(ep.scale_a + m));
        const float4 o = make_float4((float)acc.x * sa.x * sb, (float)acc.y * sa.y * sb, (float)acc.z * sa.z * sb,
                                     (float)acc.w * sa.w * sb);
        store_four(ep, (long long)n * ep.ldo + m, n, m, o);
      } else {
        const int a4[4] = {acc.x, acc.y, acc.z, acc.w};
        for (int j = 0; j < 4 && m + j < M; ++j) store_one(ep, m + j, n, (float)a4[j] * __ldg(ep.scale_a + m + j) * sb);
      }
    }
  } else {
    // output (m, n) at out[m * ldo + n]: vectors of 4 consecutive n of one row m
    const int per_row = BN / 4;
    for (int v = e; v < R * per_row; v += 128) {
      const int row = r0 + v / per_row, c4 = 4 * (v % per_row);
      const int m = m0 + row, n = n0 + c4;
      if (m >= M || n >= N) continue;
      const uint32_t a = base + (uint32_t)(row * CS + c4) * 4u;
      int4 acc = sm100::ld_dsmem_v4(sm100::mapa(a, 0));
      for (int q = 1; q < S; ++q) {
        const int4 x = sm100::ld_dsmem_v4(sm100::mapa(a, q));
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
      const float sa = __ldg(ep.scale_a + m);
      if (n + 3 < N && (vec_ok || ep.mode == 5) && (reinterpret_cast<uintptr_t>(ep.scale_b + n) & 15) == 0) {
        const float4 sb = __ldg(reinterpret_cast<const float4*>(ep.scale_b + n));
        const float4 o = make_float4((float)acc.x * sa * sb.x, (float)acc.y * sa * sb.y, (float)acc.z * sa * sb.z,
                                     (float)acc.w * sa * sb.w);
        store_four(ep, (long long)m * ep.ldo + n, m, n, o);
      } else {
        const int a4[4] = {acc.x, acc.y, acc.z, acc.w};
        for (int j = 0; j < 4 && n + j < N; ++j) store_one(ep, m, n + j, (float)a4[j] * sa * __ldg(ep.scale_b + n + j));
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               GemmEpi ep, int M, int N, int K, int splits, int* status) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int k_blocks = (K + BK - 1) / BK;
  const int kb_per_split = (k_blocks + splits - 1) / splits;
  const int total = m_tiles * n_tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&acc_full[a], 1);
      sm100::mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    sm100::prefetch_tmap(&tmA);
    sm100::prefetch_tmap(&tmB);
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Under programmatic dependent launch the set-up above overlapped the previous
  // kernel; everything below that reads or writes memory it may touch waits for it.
  // The TMA warp first fetches the static operand's first stages (below).
  if (warp != 0) sm100::griddep_wait();
  // the next kernel, if it is a programmatic dependent (another GEMM), may place its
  // CTAs on SMs this grid leaves free and prefetch its weights there
  sm100::griddep_launch_dependents();

  auto tile_coords = [&](int t, int& m0, int& n0, int& kb0, int& kb1) {
    const int split = t % splits;
    const int mn = t / splits;
    // n-major traversal keeps consecutive CTAs on the same A rows (weights in
    // swapped mode) so they share L2.
    const int mt = mn % m_tiles, nt = mn / m_tiles;
    m0 = mt * BM;
    n0 = nt * BN;
    kb0 = split * kb_per_split;
    kb1 = min(k_blocks, kb0 + kb_per_split);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (sm100::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_parity = 0;  // per stage: a copy was issued, with this phase
      // The weights (the static operand) of the first tile's first stages are fetched
      // before waiting for the previous kernel: they do not depend on it, and the
      // fetch overlaps its tail.  Those stages are fresh, so no `empty` wait is needed.
      const bool pre_a = ep.a_static != 0, pre_b = !pre_a && ep.b_static != 0;
      int pre = 0;
      if ((pre_a || pre_b) && (int)blockIdx.x < total) {
        int m0, n0, kb0, kb1;
        tile_coords(blockIdx.x, m0, n0, kb0, kb1);
        pre = kb1 - kb0 < C::STAGES ? kb1 - kb0 : C::STAGES;
        for (int i = 0; i < pre; ++i) {
          uint8_t* sa = smem + i * C::STAGE_BYTES;
          sm100::mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          if (pre_a)
            sm100::tma_load_2d(sa, &tmA, &full[i], (kb0 + i) * BK, m0);
          else
            sm100::tma_load_2d(sa + C::A_BYTES, &tmB, &full[i], (kb0 + i) * BK, n0);
          issued_mask |= 1u << i;
        }
      }
      sm100::griddep_wait();
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m0, n0, kb0, kb1;
        tile_coords(t, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          if (pre > 0) {  // static half already in flight: add the dependent half
            --pre;
            if (!pre_a) sm100::tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
            if (pre_a) sm100::tma_load_2d(sb, &tmB, &full[stage], kb * BK, n0);
            if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
            continue;
          }
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kTimeoutSlotEmpty, kWaitBudgetNs)) {
            ok = false;
            break;
          }
          sm100::mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          sm100::tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
          sm100::tma_load_2d(sb, &tmB, &full[stage], kb * BK, n0);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // Aborted: let every copy already issued land (bounded) before the CTA
        // retires its shared memory.
        const uint64_t t0 = globaltimer_ns();
        for (int s = 0; s < C::STAGES; ++s) {
          if (!(issued_mask >> s & 1)) continue;
          while (!sm100::mbar_try_wait(&full[s], (issued_parity >> s) & 1)) {
            if (globaltimer_ns() - t0 > 200000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = sm100::idesc_i8(BM, BN);
    if (sm100::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
        int m0, n0, kb0, kb1;
        tile_coords(t, m0, n0, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!sm100::mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, status, kTimeoutAccEmpty, kWaitBudgetNs)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!sm100::mbar_wait(&full[stage], phase, abort_flag, status, kTimeoutTmaFull, kWaitBudgetNs)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint8_t* sa = smem + stage * C::STAGE_BYTES;
          const uint8_t* sb = sa + C::A_BYTES;
          const uint64_t da = sm100::smem_desc_sw128(sa);
          const uint64_t db = sm100::smem_desc_sw128(sb);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // Advance along K inside the 128 B swizzle row: +32 B == +2 in the
            // descriptor's 16-byte address units.
            sm100::umma_i8(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          sm100::umma_commit(&empty[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        sm100::umma_commit(&acc_full[acc]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. 32*quarter+31
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      int m0, n0, kb0, kb1;
      tile_coords(t, m0, n0, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!sm100::mbar_wait(&acc_full[acc], acc_phase, abort_flag, status, kTimeoutAccFull, kWaitBudgetNs)) break;
      sm100::tc_fence_after();
      if (ep.cluster_k > 1) {
        // Stage this CTA's int32 partial tile in shared memory for the cluster reduction.
        // The operand ring is free: this was the CTA's only tile and its MMAs are done.
        int32_t* red = reinterpret_cast<int32_t*>(smem);
        const bool zero = kb0 >= kb1;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          sm100::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + c, r);
          sm100::tmem_ld_wait();
          if (ep.trans) {
#pragma unroll
            for (int j = 0; j < 32; ++j) red[(c + j) * (BM + 4) + row_in_tile] = zero ? 0 : (int32_t)r[j];
          } else {
            int4* dst = reinterpret_cast<int4*>(red + row_in_tile * (BN + 4) + c);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = zero ? make_int4(0, 0, 0, 0)
                            : make_int4((int)r[4 * j], (int)r[4 * j + 1], (int)r[4 * j + 2], (int)r[4 * j + 3]);
          }
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&acc_empty[acc]);
        continue;
      }
      const int m = m0 + row_in_tile;
      const bool row_ok = m < M;
      const float sa = row_ok ? ep.scale_a[m] : 0.f;
      const bool empty_split = kb0 >= kb1;
      const bool red_vec = (ep.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(ep.out) & 15) == 0;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        sm100::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + c, r);
        sm100::tmem_ld_wait();
        if (empty_split) continue;
        const int nb = n0 + c;
        if (ep.mode == 1 && red_vec && !ep.trans) {
          // fp32 accumulate with 16-byte reductions (a quarter of the L2 reduction ops); the
          // swapped layout keeps scalar reductions (a lane-quad transpose measured slower)
          if (row_ok) {
            float* dst = reinterpret_cast<float*>(ep.out) + (long long)m * ep.ldo + nb;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              if (nb + j + 3 < N) {
                const float4 sb = __ldg(reinterpret_cast<const float4*>(ep.scale_b + nb + j));
                asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + j),
                             "f"((float)(int)r[j] * sa * sb.x), "f"((float)(int)r[j + 1] * sa * sb.y),
                             "f"((float)(int)r[j + 2] * sa * sb.z), "f"((float)(int)r[j + 3] * sa * sb.w)
                             : "memory");
              } else {
                for (int e = 0; e < 4 && nb + j + e < N; ++e)
                  atomicAdd(dst + j + e, (float)(int)r[j + e] * sa * ep.scale_b[nb + j + e]);
              }
            }
          }
          continue;
        }
        if (ep.mode == 5 && splits == 1 && !ep.trans) {
          // reduce-scatter of whole-K prefill tiles: 16-byte stores of this thread's row
          if (row_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              if (nb + j + 3 < N) {
                const float4 sb = __ldg(reinterpret_cast<const float4*>(ep.scale_b + nb + j));
                red_to_owner(ep, m, nb + j,
                             make_float4((float)(int)r[j] * sa * sb.x, (float)(int)r[j + 1] * sa * sb.y,
                                         (float)(int)r[j + 2] * sa * sb.z, (float)(int)r[j + 3] * sa * sb.w));
              } else {
                for (int e = 0; e < 4 && nb + j + e < N; ++e)
                  red_to_owner1(ep, m, nb + j + e, (float)(int)r[j + e] * sa * ep.scale_b[nb + j + e]);
              }
            }
          }
          continue;
        }
        if (!row_ok) continue;
        if (ep.mode == 0 && !ep.trans && nb + 32 <= N && (ep.ldo % 8) == 0 &&
            (reinterpret_cast<uintptr_t>(ep.out) & 15) == 0) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long long)m * ep.ldo + nb;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 v;
            v.x = pack_bf16x2((float)(int)r[j + 0] * sa * ep.scale_b[nb + j + 0], (float)(int)r[j + 1] * sa * ep.scale_b[nb + j + 1]);
            v.y = pack_bf16x2((float)(int)r[j + 2] * sa * ep.scale_b[nb + j + 2], (float)(int)r[j + 3] * sa * ep.scale_b[nb + j + 3]);
            v.z = pack_bf16x2((float)(int)r[j + 4] * sa * ep.scale_b[nb + j + 4], (float)(int)r[j + 5] * sa * ep.scale_b[nb + j + 5]);
            v.w = pack_bf16x2((float)(int)r[j + 6] * sa * ep.scale_b[nb + j + 6], (float)(int)r[j + 7] * sa * ep.scale_b[nb + j + 7]);
            *reinterpret_cast<uint4*>(o + j) = v;
          }
        } else {
          // the chunk's 32 column scales with 16-byte loads, ahead of the element loop
          float sbv[32];
          if (nb + 32 <= N && (reinterpret_cast<uintptr_t>(ep.scale_b + nb) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 f = __ldg(reinterpret_cast<const float4*>(ep.scale_b + nb + j));
              sbv[j] = f.x;
              sbv[j + 1] = f.y;
              sbv[j + 2] = f.z;
              sbv[j + 3] = f.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) sbv[j] = nb + j < N ? __ldg(ep.scale_b + nb + j) : 0.f;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = nb + j;
            if (n >= N) break;
            const float v = (float)(int)r[j] * sa * sbv[j];
            const long long idx = ep.trans ? (long long)n * ep.ldo + m : (long long)m * ep.ldo + n;
            if (ep.mode == 0) {
              reinterpret_cast<__nv_bfloat16*>(ep.out)[idx] = __float2bfloat16(v);
            } else if (ep.mode == 1) {
              atomicAdd(reinterpret_cast<float*>(ep.out) + idx, v);
            } else if (ep.mode == 5 && splits == 1) {
              // reduce-scatter of a whole-K tile: straight to the owning rank
              red_to_owner1(ep, ep.trans ? n : m, ep.trans ? m : n, v);
            } else if (ep.mode >= 3) {
              // stage in the local workspace; the reduction through the switch (mode 3),
              // the bf16 store (mode 4) or the reduce-scatter into the owning rank (mode 5)
              // is issued below with 16-byte reads
              if (splits > 1)
                atomicAdd(ep.ws + idx, v);
              else
                ep.ws[idx] = v;
            } else {
              reinterpret_cast<float*>(ep.out)[idx] = v;
            }
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&acc_empty[acc]);
      if (ep.mode >= 3 && !(ep.mode == 5 && splits == 1)) {
        // The rows of this (tile, row quarter) are complete in the workspace once every
        // split has added its part (split-K: counted in tile_cnt; else this warp alone).
        // The last contributor reads them back from L2 and reduces them into every rank
        // through the switch, 16 bytes per multimem.red, then clears the workspace.
        bool last = true;
        __threadfence();
        __syncwarp();
        const int slot = (t / splits) * 4 + quarter;
        if (splits > 1) {
          int prev = 0;
          if (lane == 0) prev = atomicAdd(ep.tile_cnt + slot, 1);
          prev = __shfl_sync(0xffffffffu, prev, 0);
          last = prev == splits - 1;
          if (last) __threadfence();
        }
        if (last) {
          // Read back the summed rows in batches of eight independent 16-byte loads
          // (one dependent load per iteration would serialise on the L2 latency).
          float* out = reinterpret_cast<float*>(ep.out);
          auto emit4 = [&](long long base, int tok, int col, const float4& v) {
            if (ep.mode == 5) {
              red_to_owner(ep, tok, col, v);
            } else if (ep.mode == 4) {
              *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(ep.out) + base) =
                  make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
            } else {
              asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(out + base),
                           "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                           : "memory");
            }
            *reinterpret_cast<float4*>(ep.ws + base) = make_float4(0.f, 0.f, 0.f, 0.f);
          };
          auto emit1 = [&](long long base, int tok, int col) {
            const float v = __ldcg(ep.ws + base);
            if (ep.mode == 5)
              red_to_owner1(ep, tok, col, v);
            else if (ep.mode == 4)
              reinterpret_cast<__nv_bfloat16*>(ep.out)[base] = __float2bfloat16(v);
            else
              asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(out + base), "f"(v) : "memory");
            ep.ws[base] = 0.f;
          };
          const int mq = m0 + quarter * 32;  // first row of this warp
          const int ncols = N - n0 < BN ? N - n0 : BN;
          if (ep.trans) {
            // element (m, n) at n * ldo + m: lanes cover 8 x 4 consecutive rows of 4 columns
            const int m4 = mq + 4 * (lane & 7);
            const bool full4 = m4 + 3 < M;
#pragma unroll 1
            for (int jb = 0; jb < ncols; jb += 32) {
              float4 v[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int jj = jb + 4 * u + (lane >> 3);
                v[u] = (jj < ncols && full4)
                           ? __ldcg(reinterpret_cast<const float4*>(ep.ws + (long long)(n0 + jj) * ep.ldo + m4))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int jj = jb + 4 * u + (lane >> 3);
                if (jj >= ncols) continue;
                const int n = n0 + jj;
                const long long base = (long long)n * ep.ldo + m4;
                if (full4) {
                  emit4(base, n, m4, v[u]);
                } else {
                  for (int e = 0; m4 + e < M && e < 4; ++e) emit1(base + e, n, m4 + e);
                }
              }
            }
          } else if (row_ok) {
            // element (m, n) at m * ldo + n: each thread owns a row
#pragma unroll 1
            for (int jb = 0; jb < ncols; jb += 32) {
              float4 v[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int j = jb + 4 * u;
                v[u] = j + 3 < ncols ? __ldcg(reinterpret_cast<const float4*>(ep.ws + (long long)m * ep.ldo + n0 + j))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int j = jb + 4 * u;
                if (j >= ncols) break;
                const long long base = (long long)m * ep.ldo + n0 + j;
                if (j + 3 < ncols) {
                  emit4(base, m, n0 + j, v[u]);
                } else {
                  for (int e = 0; j + e < ncols; ++e) emit1(base + e, m, n0 + j + e);
                }
              }
            }
          }
          __syncwarp();
          if (splits > 1 && lane == 0) ep.tile_cnt[slot] = 0;
        }
      }
    }
  }

  if (ep.cluster_k > 1) {
    // every CTA of the cluster has staged its partial tile (or aborted): reduce this
    // CTA's rows across the cluster, then keep the shared memory alive until all peers
    // have read it
    __syncwarp();
    sm100::cluster_sync();
    if (warp >= 2 && !*abort_flag) {
      int m0 = 0, n0 = 0, kb0 = 0, kb1 = 0;
      tile_coords(blockIdx.x, m0, n0, kb0, kb1);
      cluster_reduce_tile<BN>(ep, reinterpret_cast<const int32_t*>(smem), m0, n0, M, N, threadIdx.x - 64);
    }
    __syncwarp();
    sm100::cluster_sync();
  }
  if (ep.mode == 3 || ep.mode == 5) __threadfence_system();  // this thread's reductions before the done count
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if ((ep.mode == 3 || ep.mode == 5) && threadIdx.x == 0) {
    // every CTA's reductions are issued; the last CTA publishes the epoch to all ranks
    __threadfence_system();
    const int done = atomicAdd(ep.done_counter, 1) + 1;
    if (done == (int)gridDim.x) {
      __threadfence_system();
      *ep.done_counter = 0;
      const int e = *ep.epoch + 1;
      *ep.epoch = e;
      for (int q = 0; q < ep.world; ++q) {
        unsigned* slot = ep.peer_signals[q] + ep.rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slot), "r"((unsigned)e) : "memory");
      }
    }
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  long long rows, cols, ld;
  int box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.ptr);
    h ^= std::hash<long long>()(k.rows * 1315423911ll + k.cols * 2654435761ll + k.ld) + 0x9e3779b9 + (h << 6) + (h >> 2);
    return h ^ (size_t)k.box_rows;
  }
};

// 2-D int8 K-major tensor map: rows x cols (cols contiguous), row stride ld bytes.
int make_map(CUtensorMap* map, const void* ptr, long long rows, long long cols, long long ld, int box_rows) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{ptr, rows, cols, ld, box_rows};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *map = it->second;
      return 0;
    }
  }
  EncodeFn enc = get_encode();
  if (!enc) return -100;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return -101;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *map);
  return 0;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Programmatic dependent launch of the GEMM (on unless OSCAR_PDL=0): its CTAs may
// start while the previous kernel drains, set up TMEM and barriers and fetch their
// first weight tiles, then wait for that kernel before touching its outputs.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("OSCAR_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// How many CTAs of gemm_i8_kernel<BN> can be resident at once when launched in
// clusters of `S` (clusters must fit in one GPC, so this is below the SM count).
template <int BN>
int cluster_capacity(int S) {
  using C = Cfg<BN>;
  static std::mutex mu;
  static std::unordered_map<long long, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const long long key = (long long)dev * 64 + S;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (ensure_smem(gemm_i8_kernel<BN>, C::SMEM)) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_i8_kernel<BN>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n * S;
  return n * S;
}

bool cluster_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("OSCAR_GEMM_CLUSTER");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <int BN>
int pick_cluster(int tiles, int splits) {
  int S = splits < 8 ? splits : 8;
  while (S >= 2 && tiles * S > cluster_capacity<BN>(S)) --S;
  return S;
}

template <int BN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmEpi& ep, int M, int N, int K, int splits,
           int* status, cudaStream_t stream) {
  using C = Cfg<BN>;
  OSCAR_RC(ensure_smem(gemm_i8_kernel<BN>, C::SMEM));
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int total = m_tiles * n_tiles * splits;
  // cluster split-K: one CTA per (tile, K slice), the slices of a tile in one cluster
  const int grid = ep.cluster_k > 1 ? total : (total < num_sms() ? total : num_sms());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (ep.cluster_k > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = ep.cluster_k;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  OSCAR_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_i8_kernel<BN>, ta, tb, ep, M, N, K, splits, status));
  return 0;
}

}  // namespace

int run_gemm(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K, const GemmEpi& ep,
             int bn, int splits, int* status, cudaStream_t stream);
}  // namespace oscar

// A: [M, K] int8 (row stride lda bytes), B: [N, K] int8 (row stride ldb bytes).
// bn must be 32, 64, 128 or 256.  Returns 0 or an error code.
extern "C" int oscar_gemm_i8_ex(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                const float* scale_a, const float* scale_b, void* out, long long ldo, int mode,
                                int trans, int bn, int splits, int* status, int* done_counter, int* epoch,
                                unsigned** peer_signals, int rank, int world, float* ws, int* tile_cnt,
                                cudaStream_t stream, int static_ops);

extern "C" int oscar_gemm_i8(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                             const float* scale_a, const float* scale_b, void* out, long long ldo, int mode,
                             int trans, int bn, int splits, int* status, cudaStream_t stream) {
  if (mode == 3) return -105;  // the multimem mode needs the completion state: use oscar_gemm_i8_ex
  return oscar_gemm_i8_ex(A, lda, B, ldb, M, N, K, scale_a, scale_b, out, ldo, mode, trans, bn, splits, status,
                          nullptr, nullptr, nullptr, 0, 1, nullptr, nullptr, stream, trans ? 1 : 2);
}

extern "C" int oscar_gemm_i8_ex(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                const float* scale_a, const float* scale_b, void* out, long long ldo, int mode,
                                int trans, int bn, int splits, int* status, int* done_counter, int* epoch,
                                unsigned** peer_signals, int rank, int world, float* ws, int* tile_cnt,
                                cudaStream_t stream, int static_ops) {
  using namespace oscar;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 16) || (lda % 16) || (ldb % 16)) return -102;
  if (splits < 1) splits = 1;
  if (splits > 1 && mode != 1 && mode != 3 && mode != 4) return -104;  // split-K partial sums must be accumulated
  if (mode == 4 && (splits < 2 || !ws || !tile_cnt)) return -109;
  if (mode == 4 && (ldo % 4 || (reinterpret_cast<uintptr_t>(out) & 7) || (reinterpret_cast<uintptr_t>(ws) & 15)))
    return -108;
  if (mode == 3 && (!done_counter || !epoch || !peer_signals || world < 1)) return -106;
  if (mode == 3 && (!ws || !tile_cnt)) return -107;
  if (mode == 3 && (ldo % 4 || (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(ws) & 15)))
    return -108;  // 16-byte reductions need 16-byte aligned rows
  // static_ops: bit 0 = A, bit 1 = B does not depend on the previous kernel (weights)
  GemmEpi ep{scale_a, scale_b, out, ldo, mode, trans, done_counter, epoch, peer_signals, rank, world, ws, tile_cnt,
             static_ops & 1, (static_ops >> 1) & 1, nullptr, 0, 0, 0};
  return oscar::run_gemm(A, lda, B, ldb, M, N, K, ep, bn, splits, status, stream);
}

// Row-parallel GEMM whose epilogue reduce-scatters over the tensor-parallel ranks:
// the fp32 result row of token t is stored into slot `rank` (slot_stride floats apart)
// of rank (t / rows_per_rank)'s receive buffer peer_out[owner] (device array of `world`
// pointers) at row t % rows_per_rank.  Split-K slices are summed first, through the
// thread-block cluster (or this rank's zeroed workspace `ws` when the slices do not
// fit in clusters), so each value crosses NVLink once; the last CTA then bumps *epoch
// and stores it with release semantics into slot `rank` of every rank's signal pad
// (peer_signals[q] + rank).
extern "C" int oscar_gemm_i8_rs(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                const float* scale_a, const float* scale_b, int trans, int bn, int splits,
                                float* const* peer_out, int rows_per_rank, long long ldo, long long slot_stride,
                                int* done_counter, int* epoch, unsigned** peer_signals, int rank, int world, float* ws,
                                int* tile_cnt, int* status, cudaStream_t stream) {
  using namespace oscar;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 16) || (lda % 16) || (ldb % 16)) return -102;
  if (splits < 1) splits = 1;
  if (!peer_out || rows_per_rank < 1 || !done_counter || !epoch || !peer_signals || world < 1) return -110;
  if (!ws || !tile_cnt || (ldo % 4) || (reinterpret_cast<uintptr_t>(ws) & 15)) return -111;
  GemmEpi ep{scale_a, scale_b, ws, ldo, 5, trans, done_counter, epoch, peer_signals, rank, world, ws, tile_cnt,
             trans ? 1 : 0, trans ? 0 : 1, peer_out, rows_per_rank, slot_stride, 0};
  return run_gemm(A, lda, B, ldb, M, N, K, ep, bn, splits, status, stream);
}

namespace oscar {
template <int BN>
int run_bn(const CUtensorMap& ta, const CUtensorMap& tb, GemmEpi ep, int M, int N, int K, int splits, int* status,
           cudaStream_t stream) {
  // Split-K GEMMs whose slices meet in a workspace (modes 3, 4, 5) reduce through a
  // thread-block cluster instead when the tiles x slices fit on the GPU at once.  The
  // fp32 accumulate mode (1) keeps its fire-and-forget reductions into the output:
  // measured faster than the cluster's two barriers at decode sizes.
  ep.cluster_k = 0;
  if (splits > 1 && ep.mode >= 3 && cluster_enabled()) {
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int S = pick_cluster<BN>(tiles, splits);
    if (S >= 2) {
      ep.cluster_k = S;
      splits = S;
    }
  }
  return launch<BN>(ta, tb, ep, M, N, K, splits, status, stream);
}

int run_gemm(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K, const GemmEpi& ep,
             int bn, int splits, int* status, cudaStream_t stream) {
  CUtensorMap ta, tb;
  int rc = make_map(&ta, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&tb, B, N, K, ldb, bn);
  if (rc) return rc;
  switch (bn) {
    case 32: return run_bn<32>(ta, tb, ep, M, N, K, splits, status, stream);
    case 64: return run_bn<64>(ta, tb, ep, M, N, K, splits, status, stream);
    case 128: return run_bn<128>(ta, tb, ep, M, N, K, splits, status, stream);
    case 256: return run_bn<256>(ta, tb, ep, M, N, K, splits, status, stream);
    default: return -103;
  }
}
}  // namespace oscar

extern "C" int oscar_num_sms() { return oscar::num_sms(); }
