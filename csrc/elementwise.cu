// Memory-bound per-token kernels of the hybrid model.  Each one produces the
// int8 activation + per-token scale that the next W8A8 GEMM consumes, so no
// activation makes an extra round trip through HBM:
//
//   rmsnorm_quant   fp32 residual -> RMSNorm (x * (off + w)) -> bf16 rounding -> int8, scale
//   swiglu_quant    bf16 [gate | up] -> silu(gate) * up -> int8, scale
//   act_quant       bf16 -> int8, scale
//   embed           token ids -> fp32 residual rows (bf16 table)
//   argmax          per-row (value, index) of bf16 logits, vocab-parallel aware
#include <cstdlib>

#include "common.cuh"
#include "sm100.cuh"

namespace oscar {
namespace {

constexpr int kT = 256;  // threads of the argmax kernel
constexpr int kArgmaxChunk = 8192;  // logits per argmax CTA

// Vectorised row kernels: thread t owns vectors t, t + NT, ... of the row (4 fp32
// or 8 bf16 per 16-byte vector), all loaded before any arithmetic.
template <int NT>
OSCAR_DEVICE float row_absmax(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < NT / 32 ? red[l] : 0.f;
  return warp_max(t);
}
template <int NT>
OSCAR_DEVICE float row_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < NT / 32 ? red[l] : 0.f;
  return warp_sum(t);
}

OSCAR_DEVICE uint32_t pack_i8x4(float a, float b, float c, float d, float inv) {
  const uint32_t x0 = (uint8_t)quant_i8(a, inv), x1 = (uint8_t)quant_i8(b, inv);
  const uint32_t x2 = (uint8_t)quant_i8(c, inv), x3 = (uint8_t)quant_i8(d, inv);
  return x0 | (x1 << 8) | (x2 << 16) | (x3 << 24);
}

// RMSNorm of an fp32 row (with optional fused residual add) -> bf16-rounded -> int8.
// Cross-rank completion of a fused GEMM + all-reduce: wait (bounded) until every
// rank has published the current epoch into this rank's signal pad.
struct RankWait {
  const unsigned* signals;  // this rank's signal pad, slot q written by rank q
  const int* epoch;         // local epoch counter, bumped by the producing GEMM
  int world;
  int* status;
  uint64_t budget_ns;  // give up (status kTimeoutPeerFlag) after this long
};

OSCAR_DEVICE void wait_ranks(const RankWait& rw) {
  if (!rw.signals || threadIdx.x != 0) return;
  const unsigned e = (unsigned)*rw.epoch;
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < rw.world; ++q) {
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(rw.signals + q) : "memory");
      if ((int)(v - e) >= 0) break;
      if (globaltimer_ns() - t0 > rw.budget_ns) {  // report instead of hanging
        record_status(rw.status, kTimeoutPeerFlag);
        return;
      }
    }
  }
}

template <int NT, int PV>
__global__ void __launch_bounds__(NT) rmsnorm_quant_kernel(float* __restrict__ x, long long ldx,
                                                         float* __restrict__ delta, long long ldd,
                                                         const float* __restrict__ w, float off, float eps, int H,
                                                         int8_t* __restrict__ out, float* __restrict__ scale,
                                                         __nv_bfloat16* __restrict__ out_bf16, RankWait rw,
                                                         int zero_delta) {
  __shared__ float red[NT / 32];
  const int t = blockIdx.x;
  pdl_trigger();
  wait_ranks(rw);
  __syncthreads();
  const int nv = H / 4;
  float4* xr = reinterpret_cast<float4*>(x + (long long)t * ldx);
  float4* dr = delta ? reinterpret_cast<float4*>(delta + (long long)t * ldd) : nullptr;
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4 v[PV], wv[PV];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < PV; ++e) {
    const int i = threadIdx.x + e * NT;
    wv[e] = i < nv ? __ldg(wr + i) : make_float4(0.f, 0.f, 0.f, 0.f);  // in flight with the row loads
    v[e] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (dr && i < nv) {
      const float4 d = dr[i];
      v[e].x += d.x; v[e].y += d.y; v[e].z += d.z; v[e].w += d.w;
      xr[i] = v[e];  // fused residual add
      if (zero_delta) dr[i] = make_float4(0.f, 0.f, 0.f, 0.f);  // ready for the next reduction
    }
    ss += v[e].x * v[e].x + v[e].y * v[e].y + v[e].z * v[e].z + v[e].w * v[e].w;
  }
  ss = row_sum<NT>(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < PV; ++e) {
    const int i = threadIdx.x + e * NT;
    if (i < nv) {
      const float4 ww = wv[e];
      v[e].x = __bfloat162float(__float2bfloat16(v[e].x * inv * (off + ww.x)));
      v[e].y = __bfloat162float(__float2bfloat16(v[e].y * inv * (off + ww.y)));
      v[e].z = __bfloat162float(__float2bfloat16(v[e].z * inv * (off + ww.z)));
      v[e].w = __bfloat162float(__float2bfloat16(v[e].w * inv * (off + ww.w)));
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[e].x), fabsf(v[e].y)), fmaxf(fabsf(v[e].z), fabsf(v[e].w))));
      if (out_bf16) {
        uint2 b;
        b.x = pack_bf16x2(v[e].x, v[e].y);
        b.y = pack_bf16x2(v[e].z, v[e].w);
        reinterpret_cast<uint2*>(out_bf16 + (long long)t * H)[i] = b;
      }
    }
  }
  if (!out) return;
  amax = row_absmax<NT>(amax, red);
  const float qi = amax > 0.f ? 127.f / amax : 0.f;
  uint32_t* o = reinterpret_cast<uint32_t*>(out + (long long)t * H);
#pragma unroll
  for (int e = 0; e < PV; ++e) {
    const int i = threadIdx.x + e * NT;
    if (i < nv) o[i] = pack_i8x4(v[e].x, v[e].y, v[e].z, v[e].w, qi);
  }
  if (threadIdx.x == 0) scale[t] = amax > 0.f ? amax / 127.f : 1.f;
}

OSCAR_DEVICE void unpack_bf16x8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 a = __bfloat1622float2(h[k]);
    f[2 * k] = a.x;
    f[2 * k + 1] = a.y;
  }
}

// silu(gate) * up (bf16 [gate | up] row) -> bf16-rounded -> int8 (kMode 0), or plain
// bf16 row -> int8 (kMode 1).
template <int NT, int PV, int kMode>
__global__ void __launch_bounds__(NT) row_quant_kernel(const __nv_bfloat16* __restrict__ in, long long ld, int I,
                                                     int8_t* __restrict__ out, float* __restrict__ scale) {
  __shared__ float red[NT / 32];
  const int t = blockIdx.x;
  pdl_trigger();
  const int nv = I / 8;
  const uint4* g = reinterpret_cast<const uint4*>(in + (long long)t * ld);
  const uint4* u = reinterpret_cast<const uint4*>(in + (long long)t * ld + I);
  uint4 gr[PV], ur[PV];
#pragma unroll
  for (int e = 0; e < PV; ++e) {
    const int i = threadIdx.x + e * NT;
    if (i < nv) {
      gr[e] = g[i];
      if (kMode == 0) ur[e] = u[i];
    }
  }
  float amax = 0.f;
  float vals[PV][8];
#pragma unroll
  for (int e = 0; e < PV; ++e) {
    const int i = threadIdx.x + e * NT;
    if (i < nv) {
      float a[8];
      unpack_bf16x8(gr[e], a);
      if (kMode == 0) {
        float b[8];
        unpack_bf16x8(ur[e], b);
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = __bfloat162float(__float2bfloat16(silu(a[k]) * b[k]));
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        vals[e][k] = a[k];
        amax = fmaxf(amax, fabsf(a[k]));
      }
    }
  }
  amax = row_absmax<NT>(amax, red);
  const float qi = amax > 0.f ? 127.f / amax : 0.f;
  uint2* o = reinterpret_cast<uint2*>(out + (long long)t * I);
#pragma unroll
  for (int e = 0; e < PV; ++e) {
    const int i = threadIdx.x + e * NT;
    if (i < nv) {
      uint2 q;
      q.x = pack_i8x4(vals[e][0], vals[e][1], vals[e][2], vals[e][3], qi);
      q.y = pack_i8x4(vals[e][4], vals[e][5], vals[e][6], vals[e][7], qi);
      o[i] = q;
    }
  }
  if (threadIdx.x == 0) scale[t] = amax > 0.f ? amax / 127.f : 1.f;
}

__global__ void embed_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ table, int H,
                             int vocab_begin, int vocab_end, float* __restrict__ out) {
  const int t = blockIdx.x;
  const int id = tok[t];
  const bool mine = id >= vocab_begin && id < vocab_end;
  const __nv_bfloat16* row = table + (long long)(id - vocab_begin) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[(long long)t * H + i] = mine ? __bfloat162float(row[i]) : 0.f;
}

// Row argmax with ties broken toward the lowest index (torch.argmax semantics).
// Grid (rows, chunks): CTA (t, c) scans columns [c * chunk, (c + 1) * chunk) of row t and
// writes its (max, lowest index of the max) to the partials [t][c]; argmax_reduce_kernel
// then combines a row's chunks.  Splitting the vocabulary keeps every SM streaming logits
// at decode sizes (a few dozen rows of 31K-248K columns).
__global__ void __launch_bounds__(kT) argmax_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int V,
                                                 int chunk, float* __restrict__ part_val,
                                                 int* __restrict__ part_idx) {
  __shared__ float sv[kT / 32];
  __shared__ int si[kT / 32];
  const int t = blockIdx.x;
  const int c0 = blockIdx.y * chunk;
  const __nv_bfloat16* r = logits + (long long)t * ld + c0;
  const int base = c0;
  V = min(V - c0, chunk);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto take = [&](float x, int i) {
    if (x > bv || (x == bv && i < bi)) {
      bv = x;
      bi = i;
    }
  };
  if ((reinterpret_cast<uintptr_t>(r) & 15) == 0) {
    // 16-byte loads (8 logits), four in flight per thread; scalar tail
    const int nv = V / 8;
    const uint4* r4 = reinterpret_cast<const uint4*>(r);
    int c = threadIdx.x;
    for (; c + 3 * kT < nv; c += 4 * kT) {
      uint4 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) w[u] = __ldg(r4 + c + u * kT);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&w[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) take(__bfloat162float(h[e]), 8 * (c + u * kT) + e);
      }
    }
    for (; c < nv; c += kT) {
      const uint4 w = __ldg(r4 + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
      for (int e = 0; e < 8; ++e) take(__bfloat162float(h[e]), 8 * c + e);
    }
    for (int i = 8 * nv + threadIdx.x; i < V; i += kT) take(__bfloat162float(r[i]), i);
  } else {
    for (int i = threadIdx.x; i < V; i += kT) take(__bfloat162float(r[i]), i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    bv = l < kT / 32 ? sv[l] : -INFINITY;
    bi = l < kT / 32 ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      part_val[(long long)t * gridDim.y + blockIdx.y] = bv;
      part_idx[(long long)t * gridDim.y + blockIdx.y] = bi == 0x7fffffff ? bi : bi + base;
    }
  }
}

__global__ void argmax_reduce_kernel(const float* __restrict__ part_val, const int* __restrict__ part_idx,
                                     int chunks, int index_offset, float* __restrict__ best_val,
                                     int* __restrict__ best_idx) {
  const int t = blockIdx.x, l = threadIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = l; c < chunks; c += 32) {
    const float x = part_val[(long long)t * chunks + c];
    const int i = part_idx[(long long)t * chunks + c];
    if (x > bv || (x == bv && i < bi)) {
      bv = x;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (l == 0) {
    best_val[t] = bv;
    best_idx[t] = (bi == 0x7fffffff ? 0 : bi) + index_offset;
  }
}

// ---------------------------------------------------------------------------
// Sequence-parallel tensor parallelism: every rank owns `rows` consecutive token
// rows (from `row0`) of the fp32 residual stream.  The row-parallel GEMMs
// reduce-scatter their partial sums into the owners' receive buffers, one slot per
// source rank (GEMM epilogue mode 5); this kernel then, per owned row, waits for all
// ranks' reduce-scatter epochs, adds the slots in rank order (deterministic) into the
// residual, normalises, quantises, and writes the int8 row + scale (and the bf16 row
// when asked) into the same rows of every rank's full-height buffers - the
// all-gather, pushed over NVLink as the rows are produced.  The last CTA publishes
// this rank's all-gather epoch into slot `rank` of every rank's signal pad; the
// consumer waits for all slots (wait_flags_kernel) before the next GEMM reads.
constexpr int kMaxRanks = 8;
struct AgTargets {
  int8_t* xq[kMaxRanks];          // [rows_full, H] per rank
  float* xs[kMaxRanks];           // [rows_full] per rank
  __nv_bfloat16* hid[kMaxRanks];  // [rows_full, H] per rank, or nullptr
  unsigned* slot[kMaxRanks];      // slot `rank` of each rank's all-gather signal pad
  int world;
  int row0;   // first global row of this rank
  int rows;   // rows owned by this rank (0 allowed: the kernel still publishes)
  int* done;  // CTA completion counter, zero between launches
  int* epoch; // this rank's all-gather epoch
};

template <int NT, int PV>
__global__ void __launch_bounds__(NT) rmsnorm_ag_kernel(float* __restrict__ x, long long ldx,
                                                      const float* __restrict__ delta, long long ldd,
                                                      int n_slots, long long slot_stride,
                                                      const float* __restrict__ w, float off, float eps, int H,
                                                      RankWait rw, AgTargets ag) {
  __shared__ float red[NT / 32];
  // launched as a programmatic dependent of the reduce-scatter GEMM: resident early, it
  // touches nothing before that GEMM has completed
  sm100::griddep_wait();
  pdl_trigger();
  wait_ranks(rw);
  __syncthreads();
  const int tl = blockIdx.x;
  if (tl < ag.rows) {
    const int t = ag.row0 + tl;
    const int nv = H / 4;
    float4* xr = reinterpret_cast<float4*>(x + (long long)tl * ldx);
    const float4* dr = delta ? reinterpret_cast<const float4*>(delta + (long long)tl * ldd) : nullptr;
    const float4* wr = reinterpret_cast<const float4*>(w);
    float4 v[PV], wv[PV];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < PV; ++e) {
      const int i = threadIdx.x + e * NT;
      wv[e] = i < nv ? __ldg(wr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[e] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (dr) {
      // slots written by other GPUs: read past L1, all slots' loads in flight together
      float4 d[PV];
#pragma unroll
      for (int e = 0; e < PV; ++e) d[e] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < n_slots; ++q) {
        const float4* dq = dr + q * (slot_stride / 4);
#pragma unroll
        for (int e = 0; e < PV; ++e) {
          const int i = threadIdx.x + e * NT;
          if (i < nv) {
            const float4 a = __ldcg(dq + i);
            d[e].x += a.x; d[e].y += a.y; d[e].z += a.z; d[e].w += a.w;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < PV; ++e) {
        const int i = threadIdx.x + e * NT;
        if (i < nv) {
          v[e].x += d[e].x; v[e].y += d[e].y; v[e].z += d[e].z; v[e].w += d[e].w;
          xr[i] = v[e];
        }
      }
    }
#pragma unroll
    for (int e = 0; e < PV; ++e) ss += v[e].x * v[e].x + v[e].y * v[e].y + v[e].z * v[e].z + v[e].w * v[e].w;
    ss = row_sum<NT>(ss, red);
    const float inv = rsqrtf(ss / (float)H + eps);
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < PV; ++e) {
      const int i = threadIdx.x + e * NT;
      if (i < nv) {
        const float4 ww = wv[e];
        v[e].x = __bfloat162float(__float2bfloat16(v[e].x * inv * (off + ww.x)));
        v[e].y = __bfloat162float(__float2bfloat16(v[e].y * inv * (off + ww.y)));
        v[e].z = __bfloat162float(__float2bfloat16(v[e].z * inv * (off + ww.z)));
        v[e].w = __bfloat162float(__float2bfloat16(v[e].w * inv * (off + ww.w)));
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[e].x), fabsf(v[e].y)), fmaxf(fabsf(v[e].z), fabsf(v[e].w))));
        if (ag.hid[0]) {
          const uint2 b = make_uint2(pack_bf16x2(v[e].x, v[e].y), pack_bf16x2(v[e].z, v[e].w));
          for (int q = 0; q < ag.world; ++q) reinterpret_cast<uint2*>(ag.hid[q] + (long long)t * H)[i] = b;
        }
      }
    }
    amax = row_absmax<NT>(amax, red);
    const float qi = amax > 0.f ? 127.f / amax : 0.f;
#pragma unroll
    for (int e = 0; e < PV; ++e) {
      const int i = threadIdx.x + e * NT;
      if (i < nv) {
        const uint32_t packed = pack_i8x4(v[e].x, v[e].y, v[e].z, v[e].w, qi);
        for (int q = 0; q < ag.world; ++q) reinterpret_cast<uint32_t*>(ag.xq[q] + (long long)t * H)[i] = packed;
      }
    }
    if (threadIdx.x == 0) {
      const float sc = amax > 0.f ? amax / 127.f : 1.f;
      for (int q = 0; q < ag.world; ++q) ag.xs[q][t] = sc;
    }
  }
  // every thread's pushes are visible system-wide before the CTA counts as done
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(ag.done, 1) + 1;
    if (done == (int)gridDim.x) {
      __threadfence_system();
      *ag.done = 0;
      const int e = *ag.epoch + 1;
      *ag.epoch = e;
      for (int q = 0; q < ag.world; ++q)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ag.slot[q]), "r"((unsigned)e) : "memory");
    }
  }
}

// Waits (bounded) until every rank has published this rank's current epoch; the
// next kernel, launched as a programmatic dependent, may start meanwhile and fetch
// whatever does not depend on the wait (the GEMM's weights).
__global__ void wait_flags_kernel(RankWait rw) {
  pdl_trigger();          // the consuming GEMM may start its weight prefetch
  sm100::griddep_wait();  // the expected epoch is written by the preceding norm
  wait_ranks(rw);
}

// Programmatic dependent launch (on unless OSCAR_PDL=0): the kernel may become resident
// while its predecessor drains; it calls griddepcontrol.wait before reading anything
// that predecessor writes.
bool ew_pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("OSCAR_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ew_pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// fp32 residual rows -> bf16 (final hidden state for the lm_head / MTP head).
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, long long n, __nv_bfloat16* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16(x[i]);
}


}  // namespace
}  // namespace oscar

using namespace oscar;

#define OSCAR_PV_DISPATCH(NV, NT, CALL)              \
  do {                                                \
    const int pv = ((NV) + (NT) - 1) / (NT);          \
    if (pv <= 1) { constexpr int PV = 1; CALL; }      \
    else if (pv <= 2) { constexpr int PV = 2; CALL; } \
    else if (pv <= 3) { constexpr int PV = 3; CALL; } \
    else if (pv <= 5) { constexpr int PV = 5; CALL; } \
    else if (pv <= 8) { constexpr int PV = 8; CALL; } \
    else return -400;                                 \
  } while (0)

extern "C" int oscar_rmsnorm_quant(float* x, long long ldx, float* delta, long long ldd, const float* w,
                                   float off, float eps, int T, int H, int8_t* out, float* scale,
                                   __nv_bfloat16* out_bf16, const unsigned* signals, const int* epoch, int world,
                                   int zero_delta, int* status, long long wait_budget_ns, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 4 || ldx % 4 || (delta && ldd % 4)) return -401;
  constexpr int NT = 256;
  RankWait rw{signals, epoch, world, status, (uint64_t)(wait_budget_ns > 0 ? wait_budget_ns : 5000000000ll)};
  OSCAR_PV_DISPATCH(H / 4, NT, (rmsnorm_quant_kernel<NT, PV><<<T, NT, 0, s>>>(x, ldx, delta, ldd, w, off, eps, H, out, scale, out_bf16, rw, zero_delta)));
  return (int)cudaGetLastError();
}

// Sequence-parallel RMSNorm + all-gather (see rmsnorm_ag_kernel).  Pointer tables
// hold `world` entries; hid may be all null.
extern "C" int oscar_rmsnorm_ag(float* x, long long ldx, const float* delta, long long ldd, int n_slots,
                                long long slot_stride, const float* w, float off,
                                float eps, int H, int rows, int row0, int8_t* const* xq, float* const* xs,
                                __nv_bfloat16* const* hid, unsigned* const* slots, int world, int* done, int* epoch,
                                const unsigned* rs_signals, const int* rs_epoch, int* status, long long budget_ns,
                                cudaStream_t s) {
  if (world < 1 || world > kMaxRanks || rows < 0) return -410;
  if (H % 4 || ldx % 4 || (delta && (ldd % 4 || slot_stride % 4))) return -401;
  AgTargets ag{};
  for (int q = 0; q < world; ++q) {
    ag.xq[q] = xq[q];
    ag.xs[q] = xs[q];
    ag.hid[q] = hid ? hid[q] : nullptr;
    ag.slot[q] = slots[q];
  }
  ag.world = world;
  ag.row0 = row0;
  ag.rows = rows;
  ag.done = done;
  ag.epoch = epoch;
  constexpr int NT = 256;
  RankWait rw{rs_signals, rs_epoch, world, status, (uint64_t)(budget_ns > 0 ? budget_ns : 5000000000ll)};
  const int grid = rows > 0 ? rows : 1;
  OSCAR_PV_DISPATCH(H / 4, NT, OSCAR_RC(launch_pdl(rmsnorm_ag_kernel<NT, PV>, dim3(grid), dim3(NT), s, x, ldx, delta, ldd,
                                                   n_slots, slot_stride, w, off, eps, H, rw, ag)));
  return (int)cudaGetLastError();
}

extern "C" int oscar_wait_flags(const unsigned* signals, const int* epoch, int world, int* status, long long budget_ns,
                                cudaStream_t s) {
  RankWait rw{signals, epoch, world, status, (uint64_t)(budget_ns > 0 ? budget_ns : 5000000000ll)};
  OSCAR_RC(launch_pdl(wait_flags_kernel, dim3(1), dim3(32), s, rw));
  return (int)cudaGetLastError();
}

extern "C" int oscar_swiglu_quant(const __nv_bfloat16* gu, long long ld, int T, int I, int8_t* out, float* scale,
                                  cudaStream_t s) {
  if (T <= 0) return 0;
  if (I % 8 || ld % 8) return -401;
  constexpr int NT = 512;
  OSCAR_PV_DISPATCH(I / 8, NT, (row_quant_kernel<NT, PV, 0><<<T, NT, 0, s>>>(gu, ld, I, out, scale)));
  return (int)cudaGetLastError();
}

extern "C" int oscar_act_quant(const __nv_bfloat16* x, long long ld, int T, int K, int8_t* out, float* scale,
                               cudaStream_t s) {
  if (T <= 0) return 0;
  if (K % 8 || ld % 8) return -401;
  if (K <= 256 * 8 * 8) {
    constexpr int NT = 256;
    OSCAR_PV_DISPATCH(K / 8, NT, (row_quant_kernel<NT, PV, 1><<<T, NT, 0, s>>>(x, ld, K, out, scale)));
  } else {  // rows up to 32768 wide (e.g. the TP1 down projection's input)
    constexpr int NT = 512;
    OSCAR_PV_DISPATCH(K / 8, NT, (row_quant_kernel<NT, PV, 1><<<T, NT, 0, s>>>(x, ld, K, out, scale)));
  }
  return (int)cudaGetLastError();
}

extern "C" int oscar_embed(const int* tok, const __nv_bfloat16* table, int T, int H, int vocab_begin, int vocab_end,
                           float* out, cudaStream_t s) {
  if (T <= 0) return 0;
  embed_kernel<<<T, 256, 0, s>>>(tok, table, H, vocab_begin, vocab_end, out);
  return (int)cudaGetLastError();
}

// ws: 2 * T * ceil(V / kArgmaxChunk) 32-bit words of scratch (chunk partials).
extern "C" int oscar_argmax(const __nv_bfloat16* logits, long long ld, int T, int V, int index_offset, float* best_val,
                            int* best_idx, void* ws, cudaStream_t s) {
  if (T <= 0) return 0;
  if (V <= 0 || !ws) return -402;
  const int chunks = (V + kArgmaxChunk - 1) / kArgmaxChunk;
  float* pv = static_cast<float*>(ws);
  int* pi = reinterpret_cast<int*>(pv + (long long)T * chunks);
  argmax_kernel<<<dim3(T, chunks), kT, 0, s>>>(logits, ld, V, kArgmaxChunk, pv, pi);
  argmax_reduce_kernel<<<T, 32, 0, s>>>(pv, pi, chunks, index_offset, best_val, best_idx);
  return (int)cudaGetLastError();
}

extern "C" int oscar_f32_to_bf16(const float* x, long long n, __nv_bfloat16* y, cudaStream_t s) {
  if (n <= 0) return 0;
  int grid = (int)((n + 255) / 256);
  if (grid > 4096) grid = 4096;
  f32_to_bf16_kernel<<<grid, 256, 0, s>>>(x, n, y);
  return (int)cudaGetLastError();
}
