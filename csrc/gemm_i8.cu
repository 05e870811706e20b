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
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m0, n0, kb0, kb1;
        tile_coords(t, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kTimeoutSlotEmpty, kWaitBudgetNs)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
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
            } else if (ep.mode == 3) {
              // stage in the local workspace; the reduction through the switch is issued
              // below with 16-byte transactions
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
      if (ep.mode == 3) {
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
          float* out = reinterpret_cast<float*>(ep.out);
          const int mq = m0 + quarter * 32;  // first row of this warp
          if (ep.trans) {
            // element (m, n) at n * ldo + m: lanes cover 8 x 4 consecutive rows of 4 columns
            const int m4 = mq + 4 * (lane & 7);
            for (int jj = lane >> 3; jj < BN; jj += 4) {
              const int n = n0 + jj;
              if (n >= N) break;
              const long long base = (long long)n * ep.ldo + m4;
              if (m4 + 3 < M) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(ep.ws + base));
                asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(out + base),
                             "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                             : "memory");
                *reinterpret_cast<float4*>(ep.ws + base) = make_float4(0.f, 0.f, 0.f, 0.f);
              } else {
                for (int e = 0; e < 4 && m4 + e < M; ++e) {
                  const float v = __ldcg(ep.ws + base + e);
                  asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(out + base + e), "f"(v)
                               : "memory");
                  ep.ws[base + e] = 0.f;
                }
              }
            }
          } else if (row_ok) {
            // element (m, n) at m * ldo + n: each thread owns a row
            for (int j = 0; j < BN; j += 4) {
              const int n = n0 + j;
              if (n >= N) break;
              const long long base = (long long)m * ep.ldo + n;
              if (n + 3 < N) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(ep.ws + base));
                asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(out + base),
                             "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                             : "memory");
                *reinterpret_cast<float4*>(ep.ws + base) = make_float4(0.f, 0.f, 0.f, 0.f);
              } else {
                for (int e = 0; n + e < N; ++e) {
                  const float v = __ldcg(ep.ws + base + e);
                  asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(out + base + e), "f"(v)
                               : "memory");
                  ep.ws[base + e] = 0.f;
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

  if (ep.mode == 3) __threadfence_system();  // this thread's reductions before the CTA's done count
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (ep.mode == 3 && threadIdx.x == 0) {
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

template <int BN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmEpi& ep, int M, int N, int K, int splits,
           int* status, cudaStream_t stream) {
  using C = Cfg<BN>;
  static bool attr = false;
  if (!attr) {
    OSCAR_CUDA_CHECK(cudaFuncSetAttribute(gemm_i8_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr = true;
  }
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int total = m_tiles * n_tiles * splits;
  const int grid = total < num_sms() ? total : num_sms();
  gemm_i8_kernel<BN><<<grid, kThreads, C::SMEM, stream>>>(ta, tb, ep, M, N, K, splits, status);
  return (int)cudaGetLastError();
}

}  // namespace
}  // namespace oscar

// A: [M, K] int8 (row stride lda bytes), B: [N, K] int8 (row stride ldb bytes).
// bn must be 32, 64, 128 or 256.  Returns 0 or an error code.
extern "C" int oscar_gemm_i8_ex(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                const float* scale_a, const float* scale_b, void* out, long long ldo, int mode,
                                int trans, int bn, int splits, int* status, int* done_counter, int* epoch,
                                unsigned** peer_signals, int rank, int world, float* ws, int* tile_cnt,
                                cudaStream_t stream);

extern "C" int oscar_gemm_i8(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                             const float* scale_a, const float* scale_b, void* out, long long ldo, int mode,
                             int trans, int bn, int splits, int* status, cudaStream_t stream) {
  if (mode == 3) return -105;  // the multimem mode needs the completion state: use oscar_gemm_i8_ex
  return oscar_gemm_i8_ex(A, lda, B, ldb, M, N, K, scale_a, scale_b, out, ldo, mode, trans, bn, splits, status,
                          nullptr, nullptr, nullptr, 0, 1, nullptr, nullptr, stream);
}

extern "C" int oscar_gemm_i8_ex(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                const float* scale_a, const float* scale_b, void* out, long long ldo, int mode,
                                int trans, int bn, int splits, int* status, int* done_counter, int* epoch,
                                unsigned** peer_signals, int rank, int world, float* ws, int* tile_cnt,
                                cudaStream_t stream) {
  using namespace oscar;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 16) || (lda % 16) || (ldb % 16)) return -102;
  if (splits < 1) splits = 1;
  if (splits > 1 && mode != 1 && mode != 3) return -104;  // split-K partial sums must be accumulated
  if (mode == 3 && (!done_counter || !epoch || !peer_signals || world < 1)) return -106;
  if (mode == 3 && (!ws || !tile_cnt)) return -107;
  if (mode == 3 && (ldo % 4 || (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(ws) & 15)))
    return -108;  // 16-byte reductions need 16-byte aligned rows
  CUtensorMap ta, tb;
  int rc = make_map(&ta, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&tb, B, N, K, ldb, bn);
  if (rc) return rc;
  GemmEpi ep{scale_a, scale_b, out, ldo, mode, trans, done_counter, epoch, peer_signals, rank, world, ws, tile_cnt};
  switch (bn) {
    case 32: return launch<32>(ta, tb, ep, M, N, K, splits, status, stream);
    case 64: return launch<64>(ta, tb, ep, M, N, K, splits, status, stream);
    case 128: return launch<128>(ta, tb, ep, M, N, K, splits, status, stream);
    case 256: return launch<256>(ta, tb, ep, M, N, K, splits, status, stream);
    default: return -103;
  }
}

extern "C" int oscar_num_sms() { return oscar::num_sms(); }
