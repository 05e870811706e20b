// Launch-parameter structs shared by the CUDA kernels and the torch bindings.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace oscar {
struct GemmEpi {
  const float* scale_a;  // [M]
  const float* scale_b;  // [N]
  void* out;             // mode 3: NVLS multicast address of the fp32 reduction buffer
  long long ldo;         // elements between consecutive output rows
  int mode;              // 0: bf16 store, 1: fp32 atomic add, 2: fp32 store, 3: fp32 multimem add,
                         // 4: bf16 store of split-K partials summed in the fp32 workspace ws
                         //    (the last split of a (tile, row quarter) converts and re-zeroes),
                         // 5: reduce-scatter: fp32 row of token t stored into slot `rank` of rank
                         //    t / rows_per_rank's receive buffer peer_out[owner], at row
                         //    t % rows_per_rank (ldo floats per row, slot_stride per slot)
  int trans;             // 0: out[m * ldo + n], 1: out[n * ldo + m]
  // mode 3 completion: the last CTA bumps *epoch and stores it into slot `rank` of
  // every peer's signal pad (peer_signals[q] + rank) with release semantics.
  int* done_counter;
  int* epoch;
  unsigned** peer_signals;
  int rank, world;
  // mode 3 with split-K: partial tiles are summed in this rank's fp32 workspace
  // (same indexing as out, all zero between calls); the last split of a (tile, row
  // quarter) - counted in tile_cnt - sends the reduced rows through the switch and
  // re-zeroes them.
  float* ws;
  int* tile_cnt;
  // Operands that no earlier kernel writes (the weights): under programmatic dependent
  // launch their first tiles are fetched before the kernel waits for its predecessor.
  int a_static, b_static;
  // mode 5 (reduce-scatter): per-rank fp32 destination buffers (device array of world
  // pointers, this rank's included) and the token rows each rank owns
  float* const* peer_out;
  int rows_per_rank;
  long long slot_stride;  // mode 5: elements between the per-source-rank slots of a receive buffer
  // split-K over a thread-block cluster of cluster_k CTAs (one per K slice of a tile):
  // partial int32 tiles are summed through distributed shared memory, each CTA writes
  // BM / cluster_k rows of the result.  0 or 1: no cluster.
  int cluster_k;
};

struct StoreParams {
  const __nv_bfloat16* qkv;
  long long ld_qkv;
  int q_off, q_head_stride, k_off, v_off;
  int Hq, Hk, D;
  const float* q_norm_w;  // [D] or nullptr (no norm)
  const float* k_norm_w;
  float eps;
  float norm_offset;  // 1.0 for x * (1 + w)
  const int* positions;  // [T]
  const float* rope_cos;  // [max_pos, rot_dim/2]
  const float* rope_sin;
  int rot_dim;
  const float* Rk;  // [D, D] or nullptr (identity)
  const float* Rv;
  // Rotation split for the tensor-core path: R^T as bf16 hi + lo parts,
  // [D(n)][D(k)] each (nullptr -> SIMT fp32 path with Rk/Rv above).
  const __nv_bfloat16* RkT_hi;
  const __nv_bfloat16* RkT_lo;
  const __nv_bfloat16* RvT_hi;
  const __nv_bfloat16* RvT_lo;
  __nv_bfloat16* xbuf;  // scratch [T * (Hq + 2 Hk), D] normalised / roped rows
  int k_clip_idx, v_clip_idx;  // ascending-sort index of the clip threshold, -1 = no clip
  __half* q_out;    // [T, Hq, D]
  __half* k_fresh;  // [T, Hk, D]
  __half* v_fresh;
  int kv_mode;      // 0: INT2 pool, 1: BF16 pool (kc / vc, no quantisation)
  uint8_t* pool;    // [blocks, Hk, page_bytes]
  int page_bytes;
  __nv_bfloat16* kc;  // [blocks, 128, Hk, D]
  __nv_bfloat16* vc;
  const int* slots;  // [T]
  float* stage_k;    // [rows * 128, Hk, D]
  float* stage_v;  // [rows][Hk][D][128] (dim-major per row); stage_k: [rows * 128][Hk][D]
  const int* stage_seat;  // [T]: seat if this token is kept and wins its seat, else -1
  int* owner;             // [rows * 128]
  const int* owner_seat;  // [n_owner]
  const int* owner_val;
  int n_owner;
  int T;
  int* status;
};

struct AttnParams {
  const __half* q;  // [T, Hq, D]
  const __half* k_fresh;
  const __half* v_fresh;  // [T, Hk, D]
  int Hq, Hk, D;
  float scale;
  int kv_mode;  // 0: INT2 pool, 1: BF16 pool
  const uint8_t* pool;
  int page_bytes;
  const __nv_bfloat16* kc;  // [blocks, 128, Hk, D]
  const __nv_bfloat16* vc;
  const float* stage_k;  // [rows * 128, Hk, D]
  const float* stage_v;  // [rows][Hk][D][128]
  const int* owner;  // [rows * 128]
  int stage_rows;    // 0: staging disabled
  const int* block_tables;
  int bt_stride;
  const int* q_start;   // [R + 1]
  const int* seq_lens;  // [R]
  const int4* work;     // {req, row0, kv_begin, kv_end}
  int n_work;
  float* part_o;    // [n_work, Hk, 64, D]
  float* part_lse;  // [n_work, Hk, 64]
  int* status;
  // Staging rows per request (stage_ring > 0): logical page lp of request r uses row
  // stage_req_slot[r] * (stage_sink + stage_ring) + (lp < stage_sink ? lp
  // : stage_sink + lp % stage_ring), so the sink pages keep rows of their own and the
  // recent pages cycle through stage_ring rows.  stage_ring == 0: the hashed arena of
  // the reference (row = physical block % stage_rows).
  const int* stage_req_slot;
  int stage_sink, stage_ring;
};

#ifdef __CUDACC__
__device__ __forceinline__ int stage_row_of(const AttnParams& p, int req, int lp, int blk) {
  if (p.stage_ring > 0)
    return p.stage_req_slot[req] * (p.stage_sink + p.stage_ring) +
           (lp < p.stage_sink ? lp : p.stage_sink + lp % p.stage_ring);
  return blk % p.stage_rows;
}
#endif

struct MergeParams {
  const float* part_o;
  const float* part_lse;
  const int* item_first;  // [R * max_rb]
  const int* item_count;
  int max_rb;
  const int* tok_req;  // [T] request of each query token
  const int* q_start;  // [R + 1]
  int Hq, Hk, D;
  const float* RvT;  // [D, D] (o = o_rot @ R_v^T) or nullptr
  const __nv_bfloat16* gate;  // gate[t * gate_ld + h * gate_hstride + d] or nullptr
  long long gate_ld;
  int gate_hstride;
  __nv_bfloat16* out_bf16;  // [T, Hq * D] or nullptr
  int8_t* out_i8;           // [T, Hq * D] or nullptr
  float* out_scale;         // [T]
  int T;
};

struct GdnParams {
  const __nv_bfloat16* qkvz;  // [T, ld_qkvz]; per k-head group: q(dk) k(dk) v(r*dv) z(r*dv)
  long long ld_qkvz;
  const __nv_bfloat16* ba;  // [T, ld_ba]; per k-head group: b(r) a(r)
  long long ld_ba;
  int Hk, Hv, dk, dv;
  const float* conv_w;   // [conv_dim, 4]; channels [q heads | k heads | v heads]
  const float* A_log;    // [Hv]
  const float* dt_bias;  // [Hv]
  const float* norm_w;   // [dv]
  float eps;
  __nv_bfloat16* state;  // [slots, Hv, dk, dv]
  // The conv window and the pending raw inputs are ping-ponged per slot (buffer
  // `parity` is read, 1 - parity written): the q/k channels of a key head are
  // shared by the r value-head CTAs of that group.
  __nv_bfloat16* conv_state;  // [2, slots, conv_dim, 3] raw inputs, oldest first
  __nv_bfloat16* pend_x;      // [2, slots, P, conv_dim]
  __nv_bfloat16* pend_ba;     // [slots, P, 2 * Hv]  (b then a, per v head; owned per head)
  const int* parity;          // [R]
  int slots;
  int P;
  const int* req_slot;      // [R]
  const int* q_start;       // [R + 1]
  const int* n_commit;      // [R]
  const int* keep_pending;  // [R]
  __nv_bfloat16* out;       // [T, Hv * dv]
  int R;
  int* status;
  // Chunked (WY-form) prefill path for requests with long_min <= T tokens, nothing to
  // commit and nothing kept pending; long_min == 0 disables it.  Workspaces:
  int long_min;
  int max_chunks;             // capacity of the per-chunk workspaces (64-token chunks)
  __nv_bfloat16* ws_q;        // [T, Hk, dk]  conv + SiLU + L2-normalised q (times dk^-1/2)
  __nv_bfloat16* ws_k;        // [T, Hk, dk]  conv + SiLU + L2-normalised k
  __nv_bfloat16* ws_v;        // [T, Hv, dv]  conv + SiLU v
  float* ws_beta;             // [T, Hv]      sigmoid(b)
  float* ws_lg;               // [T, Hv]      log g
  __nv_bfloat16* ws_w;        // [chunks, Hv, 64, dk]  W = T diag(beta G) K
  __nv_bfloat16* ws_ut;       // [chunks, Hv, dv, 64]  U^T, U = T diag(beta) V
  __nv_bfloat16* ws_p;        // [chunks, Hv, 64, 64]  (G_t / G_s) q_t.k_s for s <= t
  float* ws_g;                // [chunks, Hv, 64]      cumulative log decay in the chunk
};

}  // namespace oscar
