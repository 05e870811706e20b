// Split-KV merge of the attention partials with the output rotation on the
// tensor cores:   o = (sum_s w_s O_s / sum_s w_s) @ R_v^T,   then  o *= sigmoid(gate).
//
// 16 (token, head) rows per CTA (one m16 MMA slice; a decode step's few thousand
// rows then spread over all SMs).  The combined rotated output is split into bf16
// hi + lo parts and multiplied with the bf16 hi + lo parts of R_v (three MMAs:
// hi.hi + hi.lo + lo.hi, fp32 accumulation), which matches the fp32 product of the
// reference read path (``out.float() @ R_v^T``) to ~2^-16.  The gated result is
// written as bf16; the per-token int8 quantisation for o_proj follows in the
// row-quantiser kernel.
#include "common.cuh"
#include "mma.cuh"
#include "params.h"

namespace oscar {
namespace {

constexpr int kRT = 16;
constexpr int kPartRows = 64;  // rows per work item of the split-KV partials (the attention kernels' layout)
constexpr int kD = 256;
constexpr int kThreads = 256;
constexpr int kA = 0;                    // A hi tile [kRT][256] bf16
constexpr int kALo = kRT * 512;          // A lo tile
constexpr int kB = 2 * kRT * 512;        // B chunk hi + lo: 2 x [256][64] bf16 (64 KB)
constexpr int kSmem = kB + 2 * 256 * 128;

OSCAR_DEVICE uint32_t bswz(int n, int chunk) { return n * 128 + ((chunk ^ (n & 7)) << 4); }

OSCAR_DEVICE void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
OSCAR_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 2) attn_merge_rot_kernel(MergeParams p, const __nv_bfloat16* Rv_hi,
                                                                   const __nv_bfloat16* Rv_lo) {
  extern __shared__ __align__(128) uint8_t sm[];
  pdl_trigger();
  uint8_t* ahi = sm + kA;
  uint8_t* alo = sm + kALo;
  uint8_t* bhi = sm + kB;
  uint8_t* blo = bhi + 256 * 128;
  const int Hq = p.Hq, g = p.Hq / p.Hk;
  const long long rows = (long long)p.T * Hq;
  const long long r0 = (long long)blockIdx.x * kRT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- combine the split partials: warp per row, lane per 8 dims ----
  for (int r = warp; r < kRT; r += kThreads / 32) {
    const long long gr = r0 + r;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (gr < rows) {
      const int t = (int)(gr / Hq), h = (int)(gr % Hq);
      const int req = p.tok_req[t];
      const int tt = t - p.q_start[req];
      const int hk = h / g, rr = tt * g + h % g;
      const int rb = rr / kPartRows, ri = rr % kPartRows;
      const int first = p.item_first[req * p.max_rb + rb], cnt = p.item_count[req * p.max_rb + rb];
      float mx = -INFINITY;
      for (int s = 0; s < cnt; ++s) mx = fmaxf(mx, p.part_lse[((long long)(first + s) * p.Hk + hk) * kPartRows + ri]);
      float wsum = 0.f;
      if (mx > -INFINITY) {
        for (int s = 0; s < cnt; ++s) {
          const long long base = ((long long)(first + s) * p.Hk + hk) * kPartRows + ri;
          const float wgt = __expf(p.part_lse[base] - mx);
          wsum += wgt;
          const float4* po = reinterpret_cast<const float4*>(p.part_o + base * kD + lane * 8);
          const float4 x0 = po[0], x1 = po[1];
          acc[0] = fmaf(wgt, x0.x, acc[0]); acc[1] = fmaf(wgt, x0.y, acc[1]);
          acc[2] = fmaf(wgt, x0.z, acc[2]); acc[3] = fmaf(wgt, x0.w, acc[3]);
          acc[4] = fmaf(wgt, x1.x, acc[4]); acc[5] = fmaf(wgt, x1.y, acc[5]);
          acc[6] = fmaf(wgt, x1.z, acc[6]); acc[7] = fmaf(wgt, x1.w, acc[7]);
        }
      }
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= inv;
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
      const float2 hf = __bfloat1622float2(h2);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(acc[2 * e] - hf.x, acc[2 * e + 1] - hf.y);
      hi[e] = *reinterpret_cast<const uint32_t*>(&h2);
      lo[e] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    *reinterpret_cast<uint4*>(ahi + mma::swz(r, lane)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(alo + mma::swz(r, lane)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
  // ---- o = o_rot @ R_v^T: B = R_v (rows n, K-contiguous), 64-k chunks ----
  const int wn = warp;  // the 16 rows x a 32-column slice of the 256 outputs
  float acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const uint32_t ah = smem_u32(ahi), al = smem_u32(alo), bh = smem_u32(bhi), bl = smem_u32(blo);
  for (int kc = 0; kc < 4; ++kc) {
    __syncthreads();
    for (int idx = tid; idx < 256 * 8; idx += kThreads) {
      const int n = idx >> 3, ch = idx & 7;
      cp_async16(bhi + bswz(n, ch), Rv_hi + (long long)n * kD + kc * 64 + ch * 8);
      cp_async16(blo + bswz(n, ch), Rv_lo + (long long)n * kD + kc * 64 + ch * 8);
    }
    cp_async_wait_all();
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
      const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, ach = kc * 8 + 2 * ks + (lane >> 4);
      mma::ldsm_x4(ah + mma::swz(arow, ach), a0, a1, a2, a3);
      mma::ldsm_x4(al + mma::swz(arow, ach), c0, c1, c2, c3);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int n = wn * 32 + np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int ch = 2 * ks + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        mma::ldsm_x4(bh + bswz(n, ch), b0, b1, b2, b3);
        mma::mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma::mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        mma::mma_bf16(acc[2 * np], c0, c1, c2, c3, b0, b1);
        mma::mma_bf16(acc[2 * np + 1], c0, c1, c2, c3, b2, b3);
        mma::ldsm_x4(bl + bswz(n, ch), b0, b1, b2, b3);
        mma::mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma::mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  // ---- gate and bf16 output ----
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const long long gr = r0 + (lane >> 2) + half * 8;
    if (gr >= rows) continue;
    const int t = (int)(gr / Hq), h = (int)(gr % Hq);
    __nv_bfloat16* out = p.out_bf16 + (long long)t * Hq * kD + h * kD;
    const __nv_bfloat16* gate = p.gate ? p.gate + (long long)t * p.gate_ld + (long long)h * p.gate_hstride : nullptr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = wn * 32 + j * 8 + 2 * (lane & 3);
      float v0 = acc[j][2 * half], v1 = acc[j][2 * half + 1];
      if (gate) {
        v0 *= sigmoidf_(__bfloat162float(gate[col]));
        v1 *= sigmoidf_(__bfloat162float(gate[col + 1]));
      }
      *reinterpret_cast<__nv_bfloat162*>(out + col) = __floats2bfloat162_rn(v0, v1);
    }
  }
}

}  // namespace
}  // namespace oscar

// Merge + rotation + gate into out_bf16 [T, Hq * D] (out_i8 / out_scale are not used).
extern "C" int oscar_attn_merge_rot(const oscar::MergeParams* params, const __nv_bfloat16* Rv_hi,
                                    const __nv_bfloat16* Rv_lo, cudaStream_t stream) {
  using namespace oscar;
  const MergeParams& p = *params;
  if (p.T <= 0) return 0;
  if (p.D != kD || !p.out_bf16 || !Rv_hi || !Rv_lo) return -330;
  OSCAR_RC(ensure_smem(attn_merge_rot_kernel, kSmem));
  const long long rows = (long long)p.T * p.Hq;
  const int grid = (int)((rows + kRT - 1) / kRT);
  attn_merge_rot_kernel<<<grid, kThreads, kSmem, stream>>>(p, Rv_hi, Rv_lo);
  return (int)cudaGetLastError();
}
