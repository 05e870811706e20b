// One pass over a rank's vocabulary shard of the logits for sampling and exact
// speculative verification (the host side is oscar_b200/ops/sampling.py).
//
// Per row r and vocabulary chunk c (one CTA each), over the chunk's columns v:
//   greedy rows (temperature <= 0):  best = max_v logit, id = its lowest index;
//   sampled rows:  z = logit / T,  allowed = z >= tau_r (the top-k / top-p threshold,
//   -inf when the row is not truncated),
//     m, s   = running max of allowed z and sum exp(z - m)      (online, rescaled)
//     zd     = z of the row's draft token when it is in the chunk and allowed
//     best   = max over allowed v != draft of z + Gumbel(key_r, v), id = its index,
//   with the Gumbel noise -log(-log(u)), u = ((lowbias32(key_r ^ v) >> 8) + 0.5) / 2^24,
//   key_r = lowbias32(lowbias32(seed_r) ^ pos_r)  (C. Wellons' lowbias32 hash).
// Output per (row, chunk): {m, s, zd, best, id}; the host combines chunks and ranks
// (rescaling s to the global max) and draws the acceptance of the draft.
#include "common.cuh"

namespace oscar {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 4096;  // columns per CTA

OSCAR_DEVICE uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

struct Part {
  float m, s, zd, best;
  int id;
};

// merge b into a (the sums are relative to each part's own max)
OSCAR_DEVICE void merge(Part& a, const Part& b) {
  if (b.m > a.m) {
    a.s = (a.m == -INFINITY ? 0.f : a.s * __expf(a.m - b.m)) + b.s;
    a.m = b.m;
  } else if (b.m > -INFINITY) {
    a.s += b.s * __expf(b.m - a.m);
  }
  a.zd = fmaxf(a.zd, b.zd);
  if (b.best > a.best || (b.best == a.best && b.id < a.id)) {
    a.best = b.best;
    a.id = b.id;
  }
}

OSCAR_DEVICE Part shfl_part(const Part& p, int o) {
  Part q;
  q.m = __shfl_xor_sync(0xffffffffu, p.m, o);
  q.s = __shfl_xor_sync(0xffffffffu, p.s, o);
  q.zd = __shfl_xor_sync(0xffffffffu, p.zd, o);
  q.best = __shfl_xor_sync(0xffffffffu, p.best, o);
  q.id = __shfl_xor_sync(0xffffffffu, p.id, o);
  return q;
}

__global__ void __launch_bounds__(kThreads) sample_pass_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                               int V, int vocab_begin, const float* __restrict__ temp,
                                                               const float* __restrict__ tau,
                                                               const int* __restrict__ draft,
                                                               const int* __restrict__ seed,
                                                               const int* __restrict__ pos, float* __restrict__ out) {
  __shared__ Part red[kThreads / 32];
  const int r = blockIdx.x, c = blockIdx.y;
  const int v0 = c * kChunk, v1 = min(V, v0 + kChunk);
  const float T = temp[r];
  const bool greedy = !(T > 0.f);
  const float th = tau[r];
  const int d = draft[r];
  const uint32_t key = lowbias32(lowbias32((uint32_t)seed[r]) ^ (uint32_t)pos[r]);
  const __nv_bfloat16* row = logits + (long long)r * ld;
  Part p{-INFINITY, 0.f, -INFINITY, -INFINITY, INT_MAX};
  const bool vec = (ld % 8) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0 && (v0 % 8) == 0;
  auto visit = [&](int v, float l) {
    const int gid = vocab_begin + v;
    if (greedy) {
      if (l > p.best) {  // visited in increasing v: the first maximum is kept
        p.best = l;
        p.id = gid;
      }
      return;
    }
    const float z = l / T;
    if (!(z >= th)) return;
    if (z > p.m) {
      p.s = (p.m == -INFINITY ? 0.f : p.s * __expf(p.m - z)) + 1.f;
      p.m = z;
    } else {
      p.s += __expf(z - p.m);
    }
    if (gid == d) {
      p.zd = z;
      return;
    }
    const uint32_t h = lowbias32(key ^ (uint32_t)gid);
    const float u = ((float)(h >> 8) + 0.5f) * (1.0f / 16777216.0f);
    const float sc = z + (-logf(-logf(u)));
    if (sc > p.best) {
      p.best = sc;
      p.id = gid;
    }
  };
  if (vec) {
    for (int v = v0 + 8 * threadIdx.x; v < v1; v += 8 * kThreads) {
      if (v + 8 <= v1) {
        const uint4 u = __ldcs(reinterpret_cast<const uint4*>(row + v));
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) visit(v + e, __bfloat162float(h[e]));
      } else {
        for (int e = 0; v + e < v1; ++e) visit(v + e, __bfloat162float(row[v + e]));
      }
    }
  } else {
    for (int v = v0 + threadIdx.x; v < v1; v += kThreads) visit(v, __bfloat162float(row[v]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) merge(p, shfl_part(p, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[w] = p;
  __syncthreads();
  if (threadIdx.x == 0) {
    Part a = red[0];
    for (int i = 1; i < kThreads / 32; ++i) merge(a, red[i]);
    float* o = out + ((long long)r * gridDim.y + c) * 5;
    o[0] = a.m;
    o[1] = a.s;
    o[2] = a.zd;
    o[3] = a.best;
    o[4] = a.id == INT_MAX ? -1.f : (float)a.id;
  }
}

}  // namespace
}  // namespace oscar

// logits: [n, V] bf16 with row stride ld; per-row float / int arrays of n entries;
// out: [n, chunks, 5] fp32 with chunks = ceil(V / 4096).
extern "C" int oscar_sample_pass(const __nv_bfloat16* logits, long long ld, int n, int V, int vocab_begin,
                                 const float* temp, const float* tau, const int* draft, const int* seed,
                                 const int* pos, float* out, cudaStream_t s) {
  using namespace oscar;
  if (n <= 0 || V <= 0) return 0;
  const int chunks = (V + kChunk - 1) / kChunk;
  sample_pass_kernel<<<dim3(n, chunks), kThreads, 0, s>>>(logits, ld, V, vocab_begin, temp, tau, draft, seed, pos,
                                                          out);
  return (int)cudaGetLastError();
}

extern "C" int oscar_sample_chunk() { return oscar::kChunk; }
