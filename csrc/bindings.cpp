// torch bindings of the sm_100a kernels.  Every entry point checks devices,
// dtypes and contiguity, launches on the current CUDA stream and raises on a
// launch error.  There is no CPU fallback here: the Python layer uses the
// pure-torch oracle only for CPU tensors.
#include <torch/extension.h>
#include <cstdlib>
#include <vector>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "params.h"

extern "C" {
int oscar_gemm_i8(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                  const float* scale_a, const float* scale_b, void* out, long long ldo, int mode, int trans, int bn,
                  int splits, int* status, cudaStream_t stream);
int oscar_num_sms();
int oscar_kv_store(const oscar::StoreParams* p, cudaStream_t stream);
int oscar_paged_attention(const oscar::AttnParams* p, cudaStream_t stream);
int oscar_int2_attention_tc(const oscar::AttnParams* p, int rows_per_item, cudaStream_t stream);
int oscar_attn_tc_trace(unsigned long long* buf);
int oscar_gdn_trace(unsigned long long* buf);
int oscar_mma_rate(int a_smem, int chains, int n, int iters, unsigned long long* out, cudaStream_t s);
int oscar_tmem_store_rate(int nwarps, int width, int iters, unsigned long long* out, cudaStream_t s);
int oscar_bf16_attention_tc(const oscar::AttnParams* p, long long num_blocks, int rows_per_item, cudaStream_t stream);
int oscar_attn_merge(const oscar::MergeParams* p, cudaStream_t stream);
int oscar_attn_merge_rot(const oscar::MergeParams* p, const __nv_bfloat16* Rv_hi, const __nv_bfloat16* Rv_lo,
                         cudaStream_t stream);
int oscar_gdn_step(const oscar::GdnParams* p, int smem_state, cudaStream_t stream);
int oscar_int2_prefill_tc(const oscar::AttnParams* p, const void* tiles, int n_tiles, long long fresh_rows,
                          cudaStream_t stream);
long long oscar_gdn_chunk_ws_bytes(int T, int Hk, int Hv, int max_chunks);
int oscar_gdn_chunked(oscar::GdnParams* p, int T, void* ws, cudaStream_t stream);
int oscar_rmsnorm_quant(float* x, long long ldx, float* delta, long long ldd, const float* w, float off, float eps,
                        int T, int H, int8_t* out, float* scale, __nv_bfloat16* out_bf16, const unsigned* signals,
                        const int* epoch, int world, int zero_delta, int* status, long long wait_budget_ns,
                        cudaStream_t s);
int oscar_gemm_i8_ex(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                     const float* scale_a, const float* scale_b, void* out, long long ldo, int mode, int trans, int bn,
                     int splits, int* status, int* done_counter, int* epoch, unsigned** peer_signals, int rank,
                     int world, float* ws, int* tile_cnt, cudaStream_t stream, int static_ops);
int oscar_swiglu_quant(const __nv_bfloat16* gu, long long ld, int T, int I, int8_t* out, float* scale,
                       cudaStream_t s);
int oscar_act_quant(const __nv_bfloat16* x, long long ld, int T, int K, int8_t* out, float* scale, cudaStream_t s);
int oscar_embed(const int* tok, const __nv_bfloat16* table, int T, int H, int vocab_begin, int vocab_end, float* out,
                cudaStream_t s);
int oscar_argmax(const __nv_bfloat16* logits, long long ld, int T, int V, int index_offset, float* best_val,
                 int* best_idx, void* ws, cudaStream_t s);
int oscar_f32_to_bf16(const float* x, long long n, __nv_bfloat16* y, cudaStream_t s);
int oscar_gemm_i8_rs(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                     const float* scale_a, const float* scale_b, int trans, int bn, int splits, float* const* peer_out,
                     int rows_per_rank, long long ldo, long long slot_stride, int* done_counter, int* epoch,
                     unsigned** peer_signals, int rank, int world, float* ws, int* tile_cnt, int* status,
                     cudaStream_t stream);
int oscar_rmsnorm_ag(float* x, long long ldx, const float* delta, long long ldd, int n_slots, long long slot_stride,
                     const float* w, float off, float eps, int H,
                     int rows, int row0, int8_t* const* xq, float* const* xs, __nv_bfloat16* const* hid,
                     unsigned* const* slots, int world, int* done, int* epoch, const unsigned* rs_signals,
                     const int* rs_epoch, int* status, long long budget_ns, cudaStream_t s);
int oscar_wait_flags(const unsigned* signals, const int* epoch, int world, int* status, long long budget_ns,
                     cudaStream_t s);
int oscar_sample_pass(const __nv_bfloat16* logits, long long ld, int n, int V, int vocab_begin, const float* temp,
                      const float* tau, const int* draft, const int* seed, const int* pos, float* out,
                      cudaStream_t s);
}

namespace {

using at::Tensor;
using c10::optional;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_DTYPE(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has dtype ", (x).scalar_type(), ", expected ", (dt))

template <typename T>
T* ptr(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T>
T* optr(const optional<Tensor>& t) {
  if (!(t.has_value() && t->defined())) return nullptr;
  TORCH_CHECK(t->is_cuda(), "oscar_b200: tensor operands must be CUDA tensors");
  TORCH_CHECK(t->is_contiguous(), "oscar_b200: tensor operands must be contiguous");
  return reinterpret_cast<T*>(t->data_ptr());
}
// Same, for operands the kernels index row-wise with their own stride (views allowed).
template <typename T>
T* optr_view(const optional<Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed with code ", rc,
              rc > 0 ? std::string(" (") + cudaGetErrorString((cudaError_t)rc) + ")" : std::string());
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void gemm_i8(const Tensor& A, const Tensor& B, const Tensor& scale_a, const Tensor& scale_b, Tensor& out, int64_t mode,
             int64_t trans, int64_t bn, int64_t splits, const optional<Tensor>& status) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  CHECK_DTYPE(A, at::kChar);
  CHECK_DTYPE(B, at::kChar);
  CHECK_DTYPE(scale_a, at::kFloat);
  CHECK_DTYPE(scale_b, at::kFloat);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_i8: A [M,K], B [N,K]");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_i8: K must be contiguous");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(scale_a.numel() >= M && scale_b.numel() >= N, "gemm_i8: scale sizes");
  if (mode == 0) {
    CHECK_DTYPE(out, at::kBFloat16);
  } else {
    CHECK_DTYPE(out, at::kFloat);
  }
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "gemm_i8: out must be row-major 2-D");
  if (trans) {
    TORCH_CHECK(out.size(0) >= N && out.size(1) >= M, "gemm_i8: out shape (transposed)");
  } else {
    TORCH_CHECK(out.size(0) >= M && out.size(1) >= N, "gemm_i8: out shape");
  }
  const c10::cuda::CUDAGuard guard(A.device());
  check_rc(oscar_gemm_i8(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), M, N, K, ptr<float>(scale_a),
                         ptr<float>(scale_b), out.data_ptr(), out.stride(0), (int)mode, (int)trans, (int)bn,
                         (int)splits, optr<int>(status), stream()),
           "gemm_i8");
}

// Row-parallel GEMM whose epilogue reduces into every rank's buffer through the NVLS
// multicast address `mc_ptr` (raw device address from the symmetric-memory handle),
// then publishes the completion epoch into every peer's signal pad.
void gemm_i8_allreduce(const Tensor& A, const Tensor& B, const Tensor& scale_a, const Tensor& scale_b, int64_t mc_ptr,
                       int64_t ldo, int64_t trans, int64_t bn, int64_t splits, Tensor& done_counter, Tensor& epoch,
                       int64_t peer_signals_dev, int64_t rank, int64_t world, Tensor& ws, Tensor& tile_cnt,
                       const optional<Tensor>& status) {
  CHECK_DTYPE(A, at::kChar);
  CHECK_DTYPE(B, at::kChar);
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_i8_allreduce: K must be contiguous");
  TORCH_CHECK(mc_ptr != 0 && peer_signals_dev != 0, "gemm_i8_allreduce: multicast / signal pointers required");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  const c10::cuda::CUDAGuard guard(A.device());
  check_rc(oscar_gemm_i8_ex(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), M, N, K, ptr<float>(scale_a),
                            ptr<float>(scale_b), reinterpret_cast<void*>(mc_ptr), ldo, 3, (int)trans, (int)bn,
                            (int)splits, optr<int>(status), ptr<int>(done_counter), ptr<int>(epoch),
                            reinterpret_cast<unsigned**>(peer_signals_dev), (int)rank, (int)world, ptr<float>(ws),
                            ptr<int>(tile_cnt), stream(), trans ? 1 : 2),
           "gemm_i8_allreduce");
}

// Split-K GEMM with a bf16 result: every split adds its fp32 partial into `ws` (zero
// between calls, same indexing as `out`); the last split of each (tile, row quarter),
// counted in `tile_cnt`, converts those rows to bf16 and zeroes them again.
void gemm_i8_split(const Tensor& A, const Tensor& B, const Tensor& scale_a, const Tensor& scale_b, Tensor& out,
                   int64_t trans, int64_t bn, int64_t splits, Tensor& ws, Tensor& tile_cnt,
                   const optional<Tensor>& status) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  CHECK_DTYPE(A, at::kChar);
  CHECK_DTYPE(B, at::kChar);
  CHECK_DTYPE(scale_a, at::kFloat);
  CHECK_DTYPE(scale_b, at::kFloat);
  CHECK_DTYPE(out, at::kBFloat16);
  CHECK_DTYPE(ws, at::kFloat);
  CHECK_DTYPE(tile_cnt, at::kInt);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_i8_split: A [M,K], B [N,K]");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_i8_split: K must be contiguous");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "gemm_i8_split: out must be row-major 2-D");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(scale_a.numel() >= M && scale_b.numel() >= N, "gemm_i8_split: scale sizes");
  if (trans) {
    TORCH_CHECK(out.size(0) >= N && out.size(1) >= M, "gemm_i8_split: out shape (transposed)");
  } else {
    TORCH_CHECK(out.size(0) >= M && out.size(1) >= N, "gemm_i8_split: out shape");
  }
  const long long need = trans ? (long long)(N - 1) * out.stride(0) + M : (long long)(M - 1) * out.stride(0) + N;
  TORCH_CHECK(ws.numel() >= need, "gemm_i8_split: workspace too small");
  const long long tiles = (long long)((M + 127) / 128) * ((N + bn - 1) / bn);
  TORCH_CHECK(tile_cnt.numel() >= tiles * 4, "gemm_i8_split: tile counters too small");
  const c10::cuda::CUDAGuard guard(A.device());
  check_rc(oscar_gemm_i8_ex(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), M, N, K, ptr<float>(scale_a),
                            ptr<float>(scale_b), out.data_ptr(), out.stride(0), 4, (int)trans, (int)bn, (int)splits,
                            optr<int>(status), nullptr, nullptr, nullptr, 0, 1, ptr<float>(ws), ptr<int>(tile_cnt),
                            stream(), trans ? 1 : 2),
           "gemm_i8_split");
}

// Row-parallel GEMM with the reduce-scatter epilogue (sequence-parallel TP): token row t
// of the fp32 result is added into rank t / rows_per_rank's buffer; peer_out_dev is a
// device array of `world` float pointers, peer_signals_dev one of `world` signal slots.
void gemm_i8_rs(const Tensor& A, const Tensor& B, const Tensor& scale_a, const Tensor& scale_b, int64_t trans,
                int64_t bn, int64_t splits, int64_t peer_out_dev, int64_t rows_per_rank, int64_t ldo,
                int64_t slot_stride, Tensor& done_counter, Tensor& epoch, int64_t peer_signals_dev, int64_t rank, int64_t world, Tensor& ws,
                Tensor& tile_cnt, const optional<Tensor>& status) {
  CHECK_CUDA(A);
  CHECK_DTYPE(A, at::kChar);
  CHECK_DTYPE(B, at::kChar);
  CHECK_DTYPE(ws, at::kFloat);
  CHECK_DTYPE(tile_cnt, at::kInt);
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_i8_rs: K must be contiguous");
  TORCH_CHECK(peer_out_dev != 0 && peer_signals_dev != 0, "gemm_i8_rs: peer pointer tables required");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  const long long tokens = trans ? N : M, cols = trans ? M : N;
  TORCH_CHECK(cols <= ldo && ws.numel() >= tokens * ldo, "gemm_i8_rs: workspace too small");
  TORCH_CHECK(tokens <= rows_per_rank * world, "gemm_i8_rs: more token rows than the ranks own");
  const long long tiles = (long long)((M + 127) / 128) * ((N + bn - 1) / bn);
  TORCH_CHECK(tile_cnt.numel() >= tiles * 4, "gemm_i8_rs: tile counters too small");
  const c10::cuda::CUDAGuard guard(A.device());
  check_rc(oscar_gemm_i8_rs(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), M, N, K, ptr<float>(scale_a),
                            ptr<float>(scale_b), (int)trans, (int)bn, (int)splits,
                            reinterpret_cast<float* const*>(peer_out_dev), (int)rows_per_rank, ldo, slot_stride,
                            ptr<int>(done_counter), ptr<int>(epoch), reinterpret_cast<unsigned**>(peer_signals_dev),
                            (int)rank, (int)world, ptr<float>(ws), ptr<int>(tile_cnt), optr<int>(status), stream()),
           "gemm_i8_rs");
}

// Sequence-parallel RMSNorm of this rank's `rows` residual rows with the all-gather
// pushed to every rank (pointer lists hold one raw device address per rank).
void rmsnorm_ag(Tensor& x, const optional<Tensor>& delta, int64_t n_slots, int64_t slot_stride, const Tensor& w,
                double off, double eps, int64_t rows,
                int64_t row0, const std::vector<int64_t>& xq, const std::vector<int64_t>& xs,
                const std::vector<int64_t>& hid, const std::vector<int64_t>& slots, Tensor& done, Tensor& epoch,
                int64_t rs_signals, const optional<Tensor>& rs_epoch, const optional<Tensor>& status,
                int64_t budget_ns) {
  CHECK_CUDA(x);
  CHECK_DTYPE(x, at::kFloat);
  CHECK_DTYPE(w, at::kFloat);
  const int world = (int)xq.size();
  TORCH_CHECK(world >= 1 && world <= 8 && (int)xs.size() == world && (int)slots.size() == world &&
                  (hid.empty() || (int)hid.size() == world),
              "rmsnorm_ag: one pointer per rank");
  TORCH_CHECK(x.stride(1) == 1 && x.size(0) >= rows, "rmsnorm_ag: residual rows");
  const int H = x.size(1);
  std::vector<int8_t*> pq(world);
  std::vector<float*> ps(world);
  std::vector<__nv_bfloat16*> ph(world);
  std::vector<unsigned*> psl(world);
  for (int q = 0; q < world; ++q) {
    pq[q] = reinterpret_cast<int8_t*>(xq[q]);
    ps[q] = reinterpret_cast<float*>(xs[q]);
    ph[q] = hid.empty() ? nullptr : reinterpret_cast<__nv_bfloat16*>(hid[q]);
    psl[q] = reinterpret_cast<unsigned*>(slots[q]);
  }
  float* d = optr_view<float>(delta);
  const long long ldd = d ? delta->stride(0) : 0;
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(oscar_rmsnorm_ag(ptr<float>(x), x.stride(0), d, ldd, (int)n_slots, slot_stride, ptr<float>(w), (float)off,
                            (float)eps, H, (int)rows,
                            (int)row0, pq.data(), ps.data(), hid.empty() ? nullptr : ph.data(), psl.data(), world,
                            ptr<int>(done), ptr<int>(epoch), reinterpret_cast<const unsigned*>(rs_signals),
                            optr<int>(rs_epoch), optr<int>(status), budget_ns, stream()),
           "rmsnorm_ag");
}

// Bounded wait until every rank has published this rank's current epoch into its
// signal pad slots [signals, signals + world).
void wait_flags(int64_t signals, const Tensor& epoch, int64_t world, const optional<Tensor>& status, int64_t budget_ns) {
  const c10::cuda::CUDAGuard guard(epoch.device());
  check_rc(oscar_wait_flags(reinterpret_cast<const unsigned*>(signals), ptr<int>(epoch), (int)world,
                            optr<int>(status), budget_ns, stream()),
           "wait_flags");
}

// One sampling pass over a vocabulary shard: out [n, ceil(V / 4096), 5] per row and chunk.
void sample_pass(const Tensor& logits, int64_t vocab_begin, const Tensor& temp, const Tensor& tau, const Tensor& draft,
                 const Tensor& seed, const Tensor& pos, Tensor& out) {
  CHECK_CUDA(logits);
  CHECK_DTYPE(logits, at::kBFloat16);
  CHECK_DTYPE(temp, at::kFloat);
  CHECK_DTYPE(tau, at::kFloat);
  CHECK_DTYPE(draft, at::kInt);
  CHECK_DTYPE(seed, at::kInt);
  CHECK_DTYPE(pos, at::kInt);
  CHECK_DTYPE(out, at::kFloat);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample_pass: logits [n, V] with unit column stride");
  const int n = logits.size(0), V = logits.size(1);
  TORCH_CHECK(temp.numel() >= n && tau.numel() >= n && draft.numel() >= n && seed.numel() >= n && pos.numel() >= n,
              "sample_pass: one entry per row");
  TORCH_CHECK(out.is_contiguous() && out.numel() >= (int64_t)n * ((V + 4095) / 4096) * 5, "sample_pass: out size");
  const c10::cuda::CUDAGuard guard(logits.device());
  check_rc(oscar_sample_pass(ptr<__nv_bfloat16>(logits), logits.stride(0), n, V, (int)vocab_begin, ptr<float>(temp),
                             ptr<float>(tau), ptr<int>(draft), ptr<int>(seed), ptr<int>(pos), ptr<float>(out),
                             stream()),
           "sample_pass");
}

// Install a per-CTA timeline buffer for the tcgen05 attention kernel (0 removes it).
void attn_tc_trace(int64_t ptr) { check_rc(oscar_attn_tc_trace(reinterpret_cast<unsigned long long*>(ptr)), "attn_tc_trace"); }
void gdn_trace(int64_t ptr) { check_rc(oscar_gdn_trace(reinterpret_cast<unsigned long long*>(ptr)), "gdn_trace"); }

// Tensor-core / TMEM rate microbenchmarks (one CTA on the current device): cycle counts.
std::vector<int64_t> mma_rate(int64_t a_smem, int64_t chains, int64_t n, int64_t iters) {
  auto out = at::zeros({8}, at::TensorOptions().dtype(at::kLong).device(at::kCUDA));
  check_rc(oscar_mma_rate((int)a_smem, (int)chains, (int)n, (int)iters,
                          reinterpret_cast<unsigned long long*>(out.data_ptr<int64_t>()),
                          stream()),
           "mma_rate");
  auto h = out.cpu();
  return {h[0].item<int64_t>(), h[1].item<int64_t>()};
}
std::vector<int64_t> tmem_store_rate(int64_t nwarps, int64_t width, int64_t iters) {
  auto out = at::zeros({16}, at::TensorOptions().dtype(at::kLong).device(at::kCUDA));
  check_rc(oscar_tmem_store_rate((int)nwarps, (int)width, (int)iters,
                                 reinterpret_cast<unsigned long long*>(out.data_ptr<int64_t>()),
                                 stream()),
           "tmem_store_rate");
  auto h = out.cpu();
  std::vector<int64_t> r;
  for (int w = 0; w < nwarps; ++w) r.push_back(h[w].item<int64_t>());
  return r;
}

int64_t num_sms() { return oscar_num_sms(); }

void kv_store(const Tensor& qkv, int64_t q_off, int64_t q_head_stride, int64_t k_off, int64_t v_off, int64_t Hq,
              int64_t Hk, int64_t D, const optional<Tensor>& q_norm_w, const optional<Tensor>& k_norm_w, double eps,
              double norm_offset, const Tensor& positions, const optional<Tensor>& rope_cos,
              const optional<Tensor>& rope_sin, int64_t rot_dim, const optional<Tensor>& Rk,
              const optional<Tensor>& Rv, int64_t k_clip_idx, int64_t v_clip_idx, Tensor& q_out, Tensor& k_fresh,
              Tensor& v_fresh, int64_t kv_mode, const optional<Tensor>& pool, const optional<Tensor>& kc,
              const optional<Tensor>& vc, const Tensor& slots, const optional<Tensor>& stage_k,
              const optional<Tensor>& stage_v, const optional<Tensor>& stage_seat, const optional<Tensor>& owner,
              const optional<Tensor>& owner_seat, const optional<Tensor>& owner_val, const optional<Tensor>& status,
              const optional<Tensor>& RkT_hi, const optional<Tensor>& RkT_lo, const optional<Tensor>& RvT_hi,
              const optional<Tensor>& RvT_lo, Tensor& xbuf) {
  CHECK_CUDA(qkv);
  CHECK_DTYPE(qkv, at::kBFloat16);
  TORCH_CHECK(qkv.stride(1) == 1, "qkv rows must be contiguous");
  CHECK_DTYPE(q_out, at::kHalf);
  CHECK_DTYPE(k_fresh, at::kHalf);
  CHECK_DTYPE(slots, at::kInt);
  CHECK_DTYPE(positions, at::kInt);
  CHECK_CONTIG(slots);
  CHECK_CONTIG(positions);
  CHECK_CONTIG(q_out);
  CHECK_CONTIG(k_fresh);
  CHECK_CONTIG(v_fresh);
  if (kv_mode == 0) {
    TORCH_CHECK(pool.has_value() && pool->scalar_type() == at::kByte && pool->is_contiguous(), "INT2 pool");
  } else {
    TORCH_CHECK(kc.has_value() && kc->scalar_type() == at::kBFloat16 && kc->is_contiguous(), "BF16 pool");
  }
  oscar::StoreParams p{};
  p.qkv = ptr<__nv_bfloat16>(qkv);
  p.ld_qkv = qkv.stride(0);
  p.q_off = q_off;
  p.q_head_stride = q_head_stride;
  p.k_off = k_off;
  p.v_off = v_off;
  p.Hq = Hq;
  p.Hk = Hk;
  p.D = D;
  p.q_norm_w = optr<float>(q_norm_w);
  p.k_norm_w = optr<float>(k_norm_w);
  p.eps = eps;
  p.norm_offset = norm_offset;
  p.positions = ptr<int>(positions);
  p.rope_cos = optr<float>(rope_cos);
  p.rope_sin = optr<float>(rope_sin);
  p.rot_dim = rot_dim;
  p.Rk = optr<float>(Rk);
  p.Rv = optr<float>(Rv);
  p.RkT_hi = optr<__nv_bfloat16>(RkT_hi);
  p.RkT_lo = optr<__nv_bfloat16>(RkT_lo);
  p.RvT_hi = optr<__nv_bfloat16>(RvT_hi);
  p.RvT_lo = optr<__nv_bfloat16>(RvT_lo);
  CHECK_DTYPE(xbuf, at::kBFloat16);
  CHECK_CONTIG(xbuf);
  TORCH_CHECK(xbuf.numel() >= qkv.size(0) * (Hq + 2 * Hk) * D, "kv_store: xbuf too small");
  p.xbuf = ptr<__nv_bfloat16>(xbuf);
  p.k_clip_idx = k_clip_idx;
  p.v_clip_idx = v_clip_idx;
  p.q_out = ptr<__half>(q_out);
  p.k_fresh = ptr<__half>(k_fresh);
  p.v_fresh = ptr<__half>(v_fresh);
  p.kv_mode = kv_mode;
  p.pool = optr<uint8_t>(pool);
  p.page_bytes = kv_mode == 0 ? pool->size(2) : 0;
  p.kc = optr<__nv_bfloat16>(kc);
  p.vc = optr<__nv_bfloat16>(vc);
  p.slots = ptr<int>(slots);
  p.stage_k = optr<float>(stage_k);
  p.stage_v = optr<float>(stage_v);
  p.stage_seat = optr<int>(stage_seat);
  p.owner = optr<int>(owner);
  p.owner_seat = optr<int>(owner_seat);
  p.owner_val = optr<int>(owner_val);
  p.n_owner = owner_seat.has_value() && owner_seat->defined() ? owner_seat->numel() : 0;
  p.T = qkv.size(0);
  p.status = optr<int>(status);
  const c10::cuda::CUDAGuard guard(qkv.device());
  check_rc(oscar_kv_store(&p, stream()), "kv_store");
}

void paged_attention(const Tensor& q, const Tensor& k_fresh, const Tensor& v_fresh, int64_t Hq, int64_t Hk, int64_t D,
                     double scale, int64_t kv_mode, const optional<Tensor>& pool, const optional<Tensor>& kc,
                     const optional<Tensor>& vc, const optional<Tensor>& stage_k, const optional<Tensor>& stage_v,
                     const optional<Tensor>& owner, int64_t stage_rows, const Tensor& block_tables,
                     const Tensor& q_start, const Tensor& seq_lens, const Tensor& work, Tensor& part_o,
                     Tensor& part_lse, const optional<Tensor>& status, int64_t rows_per_item,
                     const optional<Tensor>& tiles, int64_t n_tiles, int64_t n_short,
                     const optional<Tensor>& stage_req_slot, int64_t stage_sink, int64_t stage_ring) {
  CHECK_CUDA(q);
  CHECK_DTYPE(q, at::kHalf);
  CHECK_DTYPE(k_fresh, at::kHalf);
  CHECK_DTYPE(block_tables, at::kInt);
  CHECK_DTYPE(work, at::kInt);
  CHECK_CONTIG(q);
  CHECK_CONTIG(k_fresh);
  CHECK_CONTIG(v_fresh);
  CHECK_CONTIG(block_tables);
  CHECK_CONTIG(work);
  CHECK_CONTIG(q_start);
  CHECK_CONTIG(seq_lens);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(work.data_ptr()) % 16 == 0, "attention work list must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(k_fresh.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(v_fresh.data_ptr()) % 16 == 0,
              "attention q / fresh k,v must be 16-byte aligned");
  oscar::AttnParams p{};
  p.q = ptr<__half>(q);
  p.k_fresh = ptr<__half>(k_fresh);
  p.v_fresh = ptr<__half>(v_fresh);
  p.Hq = Hq;
  p.Hk = Hk;
  p.D = D;
  p.scale = scale;
  p.kv_mode = kv_mode;
  p.pool = optr<uint8_t>(pool);
  p.page_bytes = pool.has_value() && pool->defined() ? pool->size(2) : 0;
  p.kc = optr<__nv_bfloat16>(kc);
  p.vc = optr<__nv_bfloat16>(vc);
  p.stage_k = optr<float>(stage_k);
  p.stage_v = optr<float>(stage_v);
  p.owner = optr<int>(owner);
  p.stage_rows = stage_rows;
  p.block_tables = ptr<int>(block_tables);
  p.bt_stride = block_tables.stride(0);
  p.q_start = ptr<int>(q_start);
  p.seq_lens = ptr<int>(seq_lens);
  p.work = reinterpret_cast<const int4*>(work.data_ptr());
  p.n_work = work.size(0);
  p.part_o = ptr<float>(part_o);
  p.part_lse = ptr<float>(part_lse);
  p.status = optr<int>(status);
  p.stage_req_slot = optr<int>(stage_req_slot);
  p.stage_sink = (int)stage_sink;
  p.stage_ring = p.stage_req_slot ? (int)stage_ring : 0;
  TORCH_CHECK(stage_ring == 0 || (p.stage_req_slot && stage_req_slot->numel() >= q_start.numel() - 1),
              "paged_attention: the window staging layout needs one state slot per request");
  CHECK_DTYPE(part_o, at::kFloat);
  CHECK_DTYPE(part_lse, at::kFloat);
  CHECK_CONTIG(part_o);
  CHECK_CONTIG(part_lse);
  TORCH_CHECK(part_o.numel() >= (int64_t)p.n_work * Hk * 64 * D, "part_o too small");
  TORCH_CHECK(part_lse.numel() >= (int64_t)p.n_work * Hk * 64, "part_lse too small");
  const c10::cuda::CUDAGuard guard(q.device());
  // Steps with prefill ("long") requests: the planner puts the short requests' items
  // first (decode / verify, split over the KV range) and gives every 64-row block of a
  // long request one item; INT2 long requests run on the tcgen05 prefill kernel in tiles
  // of 128 rows, everything else on the warp-level kernel.
  static const bool prefill_tc = [] {
    const char* e = std::getenv("OSCAR_ATTN_PREFILL_TC");
    return !(e && e[0] == '0');
  }();
  if (n_tiles > 0 && tiles.has_value() && tiles->defined()) {
    CHECK_DTYPE((*tiles), at::kInt);
    TORCH_CHECK(tiles->is_contiguous() && reinterpret_cast<uintptr_t>(tiles->data_ptr()) % 16 == 0,
                "attention tiles must be contiguous and 16-byte aligned");
    TORCH_CHECK(n_short >= 0 && n_short <= p.n_work && n_tiles <= tiles->size(0), "attention tiles: bad counts");
    if (n_short > 0) {
      oscar::AttnParams ps = p;
      ps.n_work = (int)n_short;
      if (kv_mode == 0 && rows_per_item > 0 && rows_per_item <= 32)
        check_rc(oscar_int2_attention_tc(&ps, (int)rows_per_item, stream()), "paged_attention(tcgen05)");
      else if (kv_mode == 1 && rows_per_item > 0 && rows_per_item <= 32)
        check_rc(oscar_bf16_attention_tc(&ps, kc->size(0), (int)rows_per_item, stream()),
                 "paged_attention(bf16 tcgen05)");
      else
        check_rc(oscar_paged_attention(&ps, stream()), "paged_attention");
    }
    if (kv_mode == 0 && prefill_tc) {
      check_rc(oscar_int2_prefill_tc(&p, tiles->data_ptr(), (int)n_tiles, k_fresh.size(0), stream()),
               "paged_attention(tcgen05 prefill)");
    } else if (n_short < p.n_work) {
      oscar::AttnParams pl = p;
      pl.work = p.work + n_short;
      pl.n_work = p.n_work - (int)n_short;
      pl.part_o = p.part_o + n_short * Hk * 64 * D;
      pl.part_lse = p.part_lse + n_short * Hk * 64;
      check_rc(oscar_paged_attention(&pl, stream()), "paged_attention");
    }
    return;
  }
  // INT2 items of <= 32 rows (decode / MTP verify) run on the tcgen05 kernel
  if (kv_mode == 0 && rows_per_item > 0 && rows_per_item <= 32)
    check_rc(oscar_int2_attention_tc(&p, (int)rows_per_item, stream()), "paged_attention(tcgen05)");
  else if (kv_mode == 1 && rows_per_item > 0 && rows_per_item <= 32)
    check_rc(oscar_bf16_attention_tc(&p, kc->size(0), (int)rows_per_item, stream()), "paged_attention(bf16 tcgen05)");
  else
    check_rc(oscar_paged_attention(&p, stream()), "paged_attention");
}

void attn_merge(const Tensor& part_o, const Tensor& part_lse, const Tensor& item_first, const Tensor& item_count,
                int64_t max_rb, const Tensor& tok_req, const Tensor& q_start, int64_t Hq, int64_t Hk, int64_t D,
                const optional<Tensor>& RvT, const optional<Tensor>& gate, int64_t gate_ld, int64_t gate_hstride,
                const optional<Tensor>& out_bf16, const optional<Tensor>& out_i8, const optional<Tensor>& out_scale,
                int64_t T) {
  oscar::MergeParams p{};
  p.part_o = ptr<float>(part_o);
  p.part_lse = ptr<float>(part_lse);
  p.item_first = ptr<int>(item_first);
  p.item_count = ptr<int>(item_count);
  p.max_rb = max_rb;
  p.tok_req = ptr<int>(tok_req);
  p.q_start = ptr<int>(q_start);
  p.Hq = Hq;
  p.Hk = Hk;
  p.D = D;
  p.RvT = optr<float>(RvT);
  p.gate = optr_view<__nv_bfloat16>(gate);
  p.gate_ld = gate_ld;
  p.gate_hstride = gate_hstride;
  p.out_bf16 = optr<__nv_bfloat16>(out_bf16);
  p.out_i8 = optr<int8_t>(out_i8);
  p.out_scale = optr<float>(out_scale);
  p.T = T;
  const c10::cuda::CUDAGuard guard(part_o.device());
  check_rc(oscar_attn_merge(&p, stream()), "attn_merge");
}

void attn_merge_rot(const Tensor& part_o, const Tensor& part_lse, const Tensor& item_first,
                    const Tensor& item_count, int64_t max_rb, const Tensor& tok_req, const Tensor& q_start, int64_t Hq,
                    int64_t Hk, int64_t D, const optional<Tensor>& gate, int64_t gate_ld, int64_t gate_hstride,
                    Tensor& out_bf16, int64_t T, const Tensor& Rv_hi, const Tensor& Rv_lo) {
  CHECK_DTYPE(out_bf16, at::kBFloat16);
  CHECK_CONTIG(out_bf16);
  CHECK_DTYPE(Rv_hi, at::kBFloat16);
  CHECK_CONTIG(Rv_hi);
  CHECK_CONTIG(Rv_lo);
  oscar::MergeParams p{};
  p.part_o = ptr<float>(part_o);
  p.part_lse = ptr<float>(part_lse);
  p.item_first = ptr<int>(item_first);
  p.item_count = ptr<int>(item_count);
  p.max_rb = max_rb;
  p.tok_req = ptr<int>(tok_req);
  p.q_start = ptr<int>(q_start);
  p.Hq = Hq;
  p.Hk = Hk;
  p.D = D;
  p.gate = optr_view<__nv_bfloat16>(gate);
  p.gate_ld = gate_ld;
  p.gate_hstride = gate_hstride;
  p.out_bf16 = ptr<__nv_bfloat16>(out_bf16);
  p.T = T;
  const c10::cuda::CUDAGuard guard(part_o.device());
  check_rc(oscar_attn_merge_rot(&p, ptr<__nv_bfloat16>(Rv_hi), ptr<__nv_bfloat16>(Rv_lo), stream()), "attn_merge_rot");
}

void gdn_step(const Tensor& qkvz, const Tensor& ba, int64_t Hk, int64_t Hv, int64_t dk, int64_t dv,
              const Tensor& conv_w, const Tensor& A_log, const Tensor& dt_bias, const Tensor& norm_w, double eps,
              Tensor& state, Tensor& conv_state, Tensor& pend_x, Tensor& pend_ba, const Tensor& parity,
              const Tensor& req_slot, const Tensor& q_start, const Tensor& n_commit, const Tensor& keep_pending,
              Tensor& out, int64_t smem_state, const optional<Tensor>& status) {
  CHECK_DTYPE(qkvz, at::kBFloat16);
  CHECK_DTYPE(state, at::kBFloat16);
  CHECK_DTYPE(conv_state, at::kBFloat16);
  TORCH_CHECK(qkvz.stride(1) == 1 && ba.stride(1) == 1, "gdn_step: rows must be contiguous");
  for (const Tensor* t : std::initializer_list<const Tensor*>{&conv_w, &A_log, &dt_bias, &norm_w, &state, &conv_state, &pend_x, &pend_ba, &parity,
                          &req_slot, &q_start, &n_commit, &keep_pending, &out})
    TORCH_CHECK(t->is_contiguous(), "gdn_step: state/metadata tensors must be contiguous");
  oscar::GdnParams p{};
  p.qkvz = ptr<__nv_bfloat16>(qkvz);
  p.ld_qkvz = qkvz.stride(0);
  p.ba = ptr<__nv_bfloat16>(ba);
  p.ld_ba = ba.stride(0);
  p.Hk = Hk;
  p.Hv = Hv;
  p.dk = dk;
  p.dv = dv;
  p.conv_w = ptr<float>(conv_w);
  p.A_log = ptr<float>(A_log);
  p.dt_bias = ptr<float>(dt_bias);
  p.norm_w = ptr<float>(norm_w);
  p.eps = eps;
  p.state = ptr<__nv_bfloat16>(state);
  p.conv_state = ptr<__nv_bfloat16>(conv_state);
  p.pend_x = ptr<__nv_bfloat16>(pend_x);
  p.pend_ba = ptr<__nv_bfloat16>(pend_ba);
  p.parity = ptr<int>(parity);
  p.slots = state.size(0);
  p.P = pend_ba.size(1);
  p.req_slot = ptr<int>(req_slot);
  p.q_start = ptr<int>(q_start);
  p.n_commit = ptr<int>(n_commit);
  p.keep_pending = ptr<int>(keep_pending);
  p.out = ptr<__nv_bfloat16>(out);
  p.R = req_slot.numel();
  p.status = optr<int>(status);
  const c10::cuda::CUDAGuard guard(qkvz.device());
  // Prefill steps: requests of >= 16 new tokens (nothing to commit or keep) take the
  // chunked tensor-core path; it reads qkvz rows with 16-byte loads.
  const int T = (int)qkvz.size(0);
  const bool aligned = (p.ld_qkvz % 8 == 0) && (reinterpret_cast<uintptr_t>(p.qkvz) % 16 == 0) && dk == 128 &&
                       dv == 128;
  static const bool chunked_on = [] {
    const char* e = std::getenv("OSCAR_GDN_CHUNKED");
    return !(e && e[0] == '0');
  }();
  if (smem_state && aligned && T >= 16 && chunked_on) {
    p.long_min = 16;
    p.max_chunks = T / 64 + p.R;
    const long long bytes = oscar_gdn_chunk_ws_bytes(T, (int)Hk, (int)Hv, p.max_chunks);
    Tensor ws = at::empty({bytes}, qkvz.options().dtype(at::kByte));
    check_rc(oscar_gdn_chunked(&p, T, ws.data_ptr(), stream()), "gdn_chunked");
  }
  check_rc(oscar_gdn_step(&p, (int)smem_state, stream()), "gdn_step");
}

void rmsnorm_quant(Tensor& x, const optional<Tensor>& delta, const Tensor& w, double off, double eps,
                   const optional<Tensor>& out, const optional<Tensor>& scale, const optional<Tensor>& out_bf16,
                   int64_t signals_ptr, const optional<Tensor>& epoch, int64_t world, int64_t zero_delta,
                   const optional<Tensor>& status, int64_t wait_budget_ns) {
  CHECK_DTYPE(x, at::kFloat);
  CHECK_DTYPE(w, at::kFloat);
  TORCH_CHECK(x.stride(1) == 1, "rmsnorm_quant: rows must be contiguous");
  const bool has_d = delta.has_value() && delta->defined();
  if (has_d) TORCH_CHECK(delta->scalar_type() == at::kFloat && delta->stride(1) == 1, "delta must be fp32 rows");
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(oscar_rmsnorm_quant(ptr<float>(x), x.stride(0), optr_view<float>(delta), has_d ? delta->stride(0) : 0,
                               ptr<float>(w), off, eps, x.size(0), x.size(1), optr<int8_t>(out), optr<float>(scale),
                               optr<__nv_bfloat16>(out_bf16), reinterpret_cast<const unsigned*>(signals_ptr),
                               optr<int>(epoch), (int)world, (int)zero_delta, optr<int>(status),
                               (long long)wait_budget_ns, stream()),
           "rmsnorm_quant");
}

void swiglu_quant(const Tensor& gu, int64_t I, Tensor& out, Tensor& scale) {
  CHECK_DTYPE(gu, at::kBFloat16);
  TORCH_CHECK(gu.stride(1) == 1, "swiglu_quant: rows must be contiguous");
  const c10::cuda::CUDAGuard guard(gu.device());
  check_rc(oscar_swiglu_quant(ptr<__nv_bfloat16>(gu), gu.stride(0), gu.size(0), I, ptr<int8_t>(out),
                              ptr<float>(scale), stream()),
           "swiglu_quant");
}

void act_quant(const Tensor& x, Tensor& out, Tensor& scale) {
  CHECK_DTYPE(x, at::kBFloat16);
  TORCH_CHECK(x.stride(1) == 1, "act_quant: rows must be contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(oscar_act_quant(ptr<__nv_bfloat16>(x), x.stride(0), x.size(0), x.size(1), ptr<int8_t>(out),
                           ptr<float>(scale), stream()),
           "act_quant");
}

void embed(const Tensor& tok, const Tensor& table, int64_t vocab_begin, int64_t vocab_end, Tensor& out) {
  CHECK_DTYPE(tok, at::kInt);
  CHECK_DTYPE(table, at::kBFloat16);
  CHECK_DTYPE(out, at::kFloat);
  const c10::cuda::CUDAGuard guard(tok.device());
  check_rc(oscar_embed(ptr<int>(tok), ptr<__nv_bfloat16>(table), tok.numel(), table.size(1), vocab_begin, vocab_end,
                       ptr<float>(out), stream()),
           "embed");
}

void argmax(const Tensor& logits, int64_t index_offset, Tensor& best_val, Tensor& best_idx) {
  CHECK_DTYPE(logits, at::kBFloat16);
  TORCH_CHECK(logits.stride(1) == 1, "argmax: rows must be contiguous");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t T = logits.size(0), V = logits.size(1);
  // chunk partials (value, index) from the caching allocator: graph-capture safe
  const int64_t chunks = (V + 8191) / 8192;
  Tensor ws = at::empty({2 * T * chunks}, logits.options().dtype(at::kFloat));
  check_rc(oscar_argmax(ptr<__nv_bfloat16>(logits), logits.stride(0), (int)T, (int)V, index_offset,
                        ptr<float>(best_val), ptr<int>(best_idx), ws.data_ptr(), stream()),
           "argmax");
}

void f32_to_bf16(const Tensor& x, Tensor& y) {
  CHECK_CONTIG(x);
  CHECK_CONTIG(y);
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(oscar_f32_to_bf16(ptr<float>(x), x.numel(), ptr<__nv_bfloat16>(y), stream()), "f32_to_bf16");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "oscar_b200 sm_100a kernels";
  m.def("gemm_i8", &gemm_i8);
  m.def("attn_tc_trace", &attn_tc_trace);
  m.def("gdn_trace", &gdn_trace);
  m.def("mma_rate", &mma_rate);
  m.def("tmem_store_rate", &tmem_store_rate);
  m.def("gemm_i8_allreduce", &gemm_i8_allreduce);
  m.def("gemm_i8_split", &gemm_i8_split);
  m.def("gemm_i8_rs", &gemm_i8_rs);
  m.def("rmsnorm_ag", &rmsnorm_ag);
  m.def("wait_flags", &wait_flags);
  m.def("sample_pass", &sample_pass);
  m.def("num_sms", &num_sms);
  m.def("kv_store", &kv_store);
  m.def("paged_attention", &paged_attention);
  m.def("attn_merge", &attn_merge);
  m.def("attn_merge_rot", &attn_merge_rot);
  m.def("gdn_step", &gdn_step);
  m.def("rmsnorm_quant", &rmsnorm_quant);
  m.def("swiglu_quant", &swiglu_quant);
  m.def("act_quant", &act_quant);
  m.def("embed", &embed);
  m.def("argmax", &argmax);
  m.def("f32_to_bf16", &f32_to_bf16);
}
