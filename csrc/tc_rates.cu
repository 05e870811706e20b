// Tensor-core and tensor-memory rates on this GPU, measured by one CTA with clock64:
//  * the issue-to-completion cost of a kind::f16 tcgen05.mma (M = 128, K = 16) as a function
//    of N, of where A lives (TMEM or shared memory) and of how many independent accumulators
//    the instructions rotate over;
//  * the throughput of tcgen05.st.32x32b stores as a function of the storing warps and
//    the store width.
// These numbers decide the structure of the decode attention kernel (attention_tc.cu),
// whose MMAs are N = 32 wide (24 query rows) and whose operands are written into TMEM.
// Every wait is bounded; operands are constant fp16 tiles (their values do not matter).
#include "common.cuh"
#include "sm100.cuh"

namespace oscar {
namespace {

constexpr int kATile = 65536;    // A: 128 rows x 256 (K) fp16, K-major 128-byte swizzle
constexpr int kBTile = 131072;   // B: up to 256 rows x 256 (K) fp16
constexpr int kSmem = kATile + kBTile + 1024 + 1024;

// mode: 0 A in TMEM, 1 A in shared memory; chains: accumulators rotated over (N columns
// each, at TMEM column 256 + c * N); n: MMA N (32, 64, 128 or 256).
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int a_smem, int chains, int n, int iters,
                                                          unsigned long long* out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (sm100::smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* a_s = smem;
  uint8_t* b_s = smem + kATile;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kATile + kBTile);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kATile + kBTile + 64);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < (kATile + kBTile) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x3c003c00u, 0u, 0u, 0u);
  if (warp == 0) {
    sm100::tmem_alloc(slot, 512);
    sm100::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    sm100::mbar_init(bar, 1);
    sm100::fence_mbar_init();
  }
  sm100::fence_proxy_async();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tb = *slot;
  if (warp == 1 && lane == 0) {
    const uint32_t idq = sm100::idesc_f16(128, n, false, false);
    const uint32_t ba = sm100::smem_addr(b_s), aa = sm100::smem_addr(a_s);
    auto issue = [&](int kk, uint32_t acc_col, uint32_t acc) {
      const uint64_t bd = sm100::smem_desc(ba + (kk >> 2) * (n * 128) + (kk & 3) * 32, 16, 1024, 2);
      if (a_smem) {
        const uint64_t ad = sm100::smem_desc(aa + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024, 2);
        sm100::umma_bf16(tb + acc_col, ad, bd, idq, acc);
      } else {
        sm100::umma_f16_tmem_a(tb + acc_col, tb + kk * 8, bd, idq, acc);
      }
    };
    for (int kk = 0; kk < 16; ++kk) issue(kk, 256, kk > 0);  // warm-up
    sm100::umma_commit(bar);
    unsigned long long w = 0;
    while (!sm100::mbar_try_wait(bar, 0) && ++w < 100000000ull) {
    }
    const unsigned long long c0 = clock64();
    for (int it = 0; it < iters; ++it)
      for (int kk = 0; kk < 16; ++kk) {
        const int c = kk % chains;
        issue(kk, 256 + c * n, kk >= chains ? 1u : 0u);
      }
    const unsigned long long c1 = clock64();
    sm100::umma_commit(bar);
    w = 0;
    while (!sm100::mbar_try_wait(bar, 1) && ++w < 100000000ull) {
    }
    const unsigned long long c2 = clock64();
    out[0] = c1 - c0;
    out[1] = c2 - c0;
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tb, 512);
  }
}

// nwarps warps (<= 16) each issue `iters` stores of `width` (16, 32, 64) columns into
// their own lanes; out[w] = cycles of warp w.
__global__ void __launch_bounds__(512, 1) tmem_store_rate_kernel(int nwarps, int width, int iters,
                                                                 unsigned long long* out) {
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    sm100::tmem_alloc(&slot, 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tb = slot;
  if (warp < nwarps) {
    uint32_t a[32], b[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      a[k] = 0x3c003c00u + k;
      b[k] = k;
    }
    const uint32_t lrow = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t col0 = (warp >> 2) * 128;
    const unsigned long long c0 = clock64();
    for (int it = 0; it < iters; ++it) {
      if (width == 16)
        sm100::tmem_st_32x32b_x16(tb + lrow + col0 + (it & 7) * 16, *reinterpret_cast<const uint32_t(*)[16]>(a));
      else if (width == 32)
        sm100::tmem_st_32x32b_x32(tb + lrow + col0 + (it & 3) * 32, a);
      else
        sm100::tmem_st_32x32b_x64(tb + lrow + col0 + (it & 1) * 64, a, b);
    }
    sm100::tmem_st_wait();
    const unsigned long long c1 = clock64();
    if (lane == 0) out[warp] = c1 - c0;
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tb, 512);
  }
}

}  // namespace
}  // namespace oscar

// out[0] cycles to issue chains of 16 K-steps x iters, out[1] until their completion.
extern "C" int oscar_mma_rate(int a_smem, int chains, int n, int iters, unsigned long long* out, cudaStream_t s) {
  using namespace oscar;
  if (!(n == 32 || n == 64 || n == 128 || n == 256) || chains < 1 || chains * n > 256 || iters < 1) return -340;
  OSCAR_RC(ensure_smem(mma_rate_kernel, kSmem));
  mma_rate_kernel<<<1, 128, kSmem, s>>>(a_smem, chains, n, iters, out);
  return (int)cudaGetLastError();
}

extern "C" int oscar_tmem_store_rate(int nwarps, int width, int iters, unsigned long long* out, cudaStream_t s) {
  using namespace oscar;
  if (nwarps < 1 || nwarps > 16 || !(width == 16 || width == 32 || width == 64) || iters < 1) return -341;
  tmem_store_rate_kernel<<<1, 512, 0, s>>>(nwarps, width, iters, out);
  return (int)cudaGetLastError();
}
