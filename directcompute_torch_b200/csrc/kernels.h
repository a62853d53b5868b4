// Launch functions of libdct_cuda's kernels (internal interface, not exported).
//
// All pointers are device pointers to fp32 words (labels and counters are
// reinterpreted where noted).  Every launcher enqueues on `st` and returns the
// launch status; none of them synchronises.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace dct {

// ---- elementwise (k_elementwise.cu) ---------------------------------------
enum EwOp : int {
  EW_RELU = 0, EW_RELU6, EW_LEAKY_RELU, EW_SIGMOID, EW_EXP, EW_LOG_ABS1P, EW_TANH,
  EW_NEG, EW_ABS,
  EW_RELU_GRAD = 16, EW_RELU6_GRAD, EW_LEAKY_RELU_GRAD, EW_SIGMOID_GRAD,
  EW_ADD, EW_SUB, EW_MUL, EW_DIV, EW_MAXIMUM, EW_MINIMUM, EW_SCALE_ADD,
  // gradient helpers: masks of where maximum / minimum(a, b) routes the
  // gradient to a (a >= b resp. a <= b, or a is NaN: 1.0 else 0.0), the
  // unary ops' backward (g, saved tensor), and a broadcast copy of a
  EW_PICK_MAX = 27, EW_PICK_MIN, EW_EXP_GRAD, EW_TANH_GRAD, EW_LOG_ABS1P_GRAD, EW_FIRST,
  EW_GAP_BWD = 40,
};
// y[i] = op(x[i]) for i < n (unary ops; alpha = leaky slope)
cudaError_t launch_unary(int op, const float* x, float* y, uint64_t n, float alpha, cudaStream_t st);
// y[i] = op(a[i], b[i]) for i < n (same-shape binary ops and the *_GRAD ops,
// whose (a, b) are (upstream grad, saved forward tensor)); SCALE_ADD uses alpha, beta.
cudaError_t launch_binary_same(int op, const float* a, const float* b, float* y, uint64_t n,
                               float alpha, float beta, cudaStream_t st);
// Broadcast binary op over an N-d output (<= 8 dims, row-major, contiguous
// operands).  a_str / b_str are element strides per output dim (0 = broadcast).
cudaError_t launch_binary_bcast(int op, const float* a, const float* b, float* y, int ndim,
                                const int64_t* shape, const int64_t* a_str, const int64_t* b_str,
                                cudaStream_t st);
// C[i] = A[i] + B[i % N] (optionally ReLU'd), i < M*N.
cudaError_t launch_add_bias(const float* A, const float* B, float* C, uint64_t M, uint64_t N,
                            bool relu, cudaStream_t st);
// relu with D3D11 bounds: out[i] = i < n_in ? relu(x[i]) : 0 for i < n_out.
cudaError_t launch_relu_bounded(const float* x, uint64_t n_in, float* y, uint64_t n_out, cudaStream_t st);
// dx[i] = g[i / S] / (float)S, i < n
cudaError_t launch_gap_backward(const float* g, float* dx, uint64_t n, uint32_t S, cudaStream_t st);
// grad[r, c] = (p[r, c] - (labels[r] == c)) / B for r < rows, c < cols (K = row stride)
cudaError_t launch_softmax_ce_grad(const float* p, const float* labels, float* grad, uint32_t B,
                                   uint32_t K, uint32_t rows, uint32_t cols, cudaStream_t st);
// dst[0] += src[0]
cudaError_t launch_accumulate_scalar(const float* src, float* dst, cudaStream_t st);
// dice backward pass 2 (elementwise from per-sample sums)
cudaError_t launch_dice_grad(const float* pred, const float* target, const float* sums, float* dx,
                             uint32_t batch, uint32_t size, uint64_t n, cudaStream_t st);

// ---- reductions (k_reduce.cu) ---------------------------------------------
enum RedOp : int { RED_SUM = 0, RED_MEAN, RED_MAX, RED_ARGMAX, RED_MIN, RED_ARGMIN, RED_SUMSQ };
// Reduce x viewed as [outer, len, inner] over the middle axis.  `out` gets
// outer*inner fp32 values (sum/mean/max/min); `out_idx` (may be null) gets int32
// indices for the arg ops (and for max/min when non-null).  `scale` multiplies
// sums (1/len for mean is applied automatically).  `ws` is device scratch of
// at least reduce3d_ws_bytes(...) bytes.
size_t reduce3d_ws_bytes(int op, uint64_t outer, uint64_t len, uint64_t inner);
cudaError_t launch_reduce3d(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                            float* out, int32_t* out_idx, void* ws, cudaStream_t st);
// One shard of a reduction whose middle axis is split across ranks: instead of
// final values, one packed 8-byte partial per output (float64 sum, or float
// value << 32 | int32 index with idx_off added to the shard-local index).
// len == 0 writes identity partials.  Fold the ranks' partials, laid out
// parts[p * stride + k] (k < nout = outer*inner <= stride), with
// launch_fold_packed (merge in part order, ties to the lower index, mean
// divides by len_total).
cudaError_t launch_reduce3d_packed(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                                   int32_t idx_off, unsigned long long* packed, void* ws, cudaStream_t st);
cudaError_t launch_fold_packed(int op, const unsigned long long* parts, uint32_t nparts, uint64_t nout,
                               uint64_t stride, uint64_t len_total, float* out, int32_t* out_idx, cudaStream_t st);
// The same rank fold fused with the exchange over peer memory (dct_peer.cuh):
// put this rank's record (p.rec), wait for every rank's, fold.
struct PeerXfer;
cudaError_t launch_peer_fold_axis(int op, const PeerXfer& p, unsigned blocks, uint64_t nout, uint64_t len_total,
                                  float* out, int32_t* out_idx, cudaStream_t st);
// A whole sharded axis reduction over peer memory: the local reduction whose
// last stage (the chunk fold) also puts this rank's partials, waits for the
// peers' and folds them in rank order; a single-chunk plan instead emits the
// record into p.rec and launches launch_peer_fold_axis with `fold_blocks`.
cudaError_t launch_reduce3d_xchg(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                                 int32_t idx_off, const PeerXfer& p, uint64_t len_total, float* out,
                                 int32_t* out_idx, void* ws, unsigned fold_blocks, cudaStream_t st);
// Broadcast gradient: out (shape t) = g (shape gshape, ndim <= 8) summed over
// every dim where t has extent 1 and g does not (t right-aligned and padded
// with 1s to ndim).  float64 accumulation, rounded once.
size_t sum_to_shape_ws_bytes(int ndim, const int64_t* gshape, const int64_t* tshape);
cudaError_t launch_sum_to_shape(const float* g, int ndim, const int64_t* gshape, const int64_t* tshape,
                                float* out, void* ws, size_t ws_bytes, cudaStream_t st);
// Backward of bias + ReLU over [rows, cols] in one pass: dx = y > 0 ? g : 0 and
// db[c] = sum_r dx[r, c] (float64, rounded once), bit-identical to relu_grad
// followed by bias_grad.  dx may alias g.  `ws` holds relu_grad_colsum_ws_bytes.
// acc (optional): acc[c] = acc[c] + db[c] in float32, as a grad_accum after it.
size_t relu_grad_colsum_ws_bytes(uint64_t rows, uint64_t cols);
cudaError_t launch_relu_grad_colsum(const float* g, const float* y, float* dx, float* db, uint64_t rows,
                                    uint64_t cols, void* ws, size_t ws_bytes, cudaStream_t st,
                                    float* acc = nullptr);
// Forward of bias + ReLU over [rows, cols] with its column sums in one pass:
// y = max(0, x + b[c]) and col[c] = sum_r y[r, c], bit-identical to bias_relu
// followed by bias_grad over y.  y may alias x.  `ws` holds
// relu_grad_colsum_ws_bytes (the same plan).
cudaError_t launch_bias_relu_colsum(const float* x, const float* b, float* y, float* col, uint64_t rows,
                                    uint64_t cols, void* ws, size_t ws_bytes, cudaStream_t st);
// General strided form: out[o*inner + i] = reduce_l x[o*so + l*sl + i*si].
size_t reduce_strided_ws_bytes(uint64_t outer, uint64_t len, uint64_t inner, uint64_t so, uint64_t sl,
                               uint64_t si);
cudaError_t launch_reduce_strided(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                                  uint64_t so, uint64_t sl, uint64_t si, float* out, int32_t* out_idx, void* ws,
                                  size_t ws_bytes, cudaStream_t st);
// Full reduction of a flat vector; out32[0] = fp32 result, out64 (optional) = fp64 result.
// op: RED_SUM, RED_SUMSQ, RED_MAX, RED_MIN.  Two-pass, deterministic.
size_t full_reduce_ws_bytes();
cudaError_t launch_full_reduce(int op, const float* x, uint64_t n, float* out32, double* out64,
                               void* ws, cudaStream_t st);
// The same over this rank's n > 0 elements of a sharded vector, pass 2 also
// exchanging the records [value, count, valid, -] over peer memory and folding
// them in rank order (post 1: divide by the global count) into out32 / out64.
cudaError_t launch_full_reduce_xchg(int op, const float* x, uint64_t n, const PeerXfer& p, int post, float* out32,
                                    double* out64, void* ws, cudaStream_t st);
// Per-group sum of squares: part[off + g] = sum_{i in group g} x[i]^2, groups of 256.
cudaError_t launch_grad_sq_reduce(const float* g, uint64_t count, float* partials, uint64_t off,
                                  uint64_t ngroups, cudaStream_t st);
// [norm, scale] from partials: norm = sqrt(sum p), scale = norm > mx ? mx/(norm+1e-6) : 1
cudaError_t launch_grad_norm_final(const float* partials, uint64_t n, float max_norm, float* ns,
                                   cudaStream_t st);
// out[0] = sqrt(sum x^2 / n)
cudaError_t launch_rms(const float* x, uint64_t n, float* out, void* ws, cudaStream_t st);
// dice: per-sample (sum p*t, sum p, sum t); mode 0 -> sums[b*3+k], mode 1 -> loss[b].
// `ws` holds dice_ws_bytes (float64 chunk partials; 0 when a sample is one chunk).
size_t dice_ws_bytes(uint32_t batch, uint32_t size);
cudaError_t launch_dice_sums(const float* pred, const float* target, uint32_t batch, uint32_t size,
                             float* out, int mode, void* ws, size_t ws_bytes, cudaStream_t st);

// ---- softmax / cross-entropy (k_softmax.cu) ---------------------------------
struct SoftmaxCEArgs {
  const float* logits = nullptr;   // [rows, K]
  const void* labels = nullptr;    // [rows] float (reference layout) or int32
  bool labels_int32 = false;
  uint32_t rows = 0, K = 0;
  float* probs = nullptr;          // optional [rows, K]
  float* dlogits = nullptr;        // optional [rows, K] = (p - onehot) / grad_div
  float* logprobs = nullptr;       // optional [rows, K]
  float* loss = nullptr;           // optional scalar: sum_r ce_r / loss_div
  double* loss_partial = nullptr;  // optional: raw fp64 sum of ce_r (for sharded combine)
  double loss_div = 1.0;
  float grad_div = 1.0f;
  bool ref_max_init = false;       // true: max starts at -1e30 (nn_softmax.hlsl:8)
  uint32_t* err = nullptr;         // device-visible error word (bounded waits)
  // sharded: the loss fold also exchanges the records [loss sum, rows, valid, -]
  // over peer memory and writes loss = (sum over ranks) / loss_div
  const PeerXfer* xchg = nullptr;
};
size_t softmax_ce_ws_bytes(uint32_t rows, uint32_t K);
cudaError_t launch_softmax_ce(const SoftmaxCEArgs& a, void* ws, cudaStream_t st);
// reference argmax_correct: counter[0] += #rows with argmax == label (strict >, first wins)
cudaError_t launch_argmax_correct(const float* logits, const float* labels, uint32_t rows,
                                  uint32_t K, uint32_t* counter, cudaStream_t st);

// ---- optimizers (k_optim.cu) --------------------------------------------------
struct AdamParams { float step_size, beta1, beta2, eps, wd, clip; };
cudaError_t launch_adam(float* w, float* m, float* v, const float* g, uint64_t n,
                        const AdamParams& p, cudaStream_t st);
cudaError_t launch_sgd(float* w, const float* g, uint64_t n, float lr, float clip, cudaStream_t st);
// w -= lr * g * ns[1]   (scale read on the device)
cudaError_t launch_sgd_clipped(float* w, const float* g, uint64_t n, float lr, const float* ns,
                               cudaStream_t st);
// multi-tensor variants: one launch over a table of tensors
struct MtTensor { float* w; const float* g; float* m; float* v; uint64_t n; };
cudaError_t launch_mt_sgd(const MtTensor* t, int count, float lr, float clip, const float* ns,
                          cudaStream_t st);
cudaError_t launch_mt_adam(const MtTensor* t, int count, const AdamParams& p, cudaStream_t st);
// one fp64 partial per block; `nparts` must be >= mt_sumsq_blocks(t, count)
cudaError_t launch_mt_sumsq(const MtTensor* t, int count, double* partials, int nparts, cudaStream_t st);
uint64_t mt_sumsq_blocks(const MtTensor* t, int count);
cudaError_t launch_norm_scale_from_parts(const double* partials, int nparts, float max_norm,
                                         float* ns, cudaStream_t st);

// ---- batchnorm (k_batchnorm.cu) -------------------------------------------------
// Per-(n, c) plane partial sums into ws: stats mode: (sum x, sum x^2);
// backward mode: (sum dy, sum dy*x).  Planes are N*C, each S contiguous floats.
size_t bn_ws_bytes(uint32_t N, uint32_t C);
cudaError_t launch_bn_plane_sums(const float* x, const float* dy, uint32_t N, uint32_t C, uint32_t S,
                                 double* plane_sums, cudaStream_t st);
// Fold plane partials over n into per-channel fp64 sums: chan[c*2+k].
cudaError_t launch_bn_fold(const double* plane_sums, uint32_t N, uint32_t C, double* chan,
                           cudaStream_t st);
// The same for a sharded batch, also exchanging the records [2C sums][count,
// valid, 2C, -] over peer memory: out[0, 2C) = the sums over ranks in rank
// order, out[2C] = the global count.
cudaError_t launch_bn_fold_xchg(const double* plane_sums, uint32_t N, uint32_t C, const PeerXfer& p, double* out,
                                cudaStream_t st);
// Finalize the forward statistics from per-channel (sum, sumsq) over cnt elements.
// cnt_dev (optional): element count per channel read on the device instead of
// `cnt` (a count combined across ranks)
cudaError_t launch_bn_stats_final(const double* chan, uint32_t C, double cnt, float* mean,
                                  float* var, float* rmean, float* rvar, bool training,
                                  float momentum, cudaStream_t st, const double* cnt_dev = nullptr);
// Finalize backward: dgamma = (sum dy*x - mean*sum dy) * rstd, dbeta = sum dy.
cudaError_t launch_bn_bwd_final(const double* chan, uint32_t C, const float* mean, const float* var,
                                float eps, float* dgamma, float* dbeta, cudaStream_t st);
cudaError_t launch_bn_forward(const float* x, const float* mean, const float* var, const float* gamma,
                              const float* beta, float* y, uint32_t N, uint32_t C, uint32_t S,
                              float eps, uint64_t limit, cudaStream_t st);
cudaError_t launch_bn_backward_dx(const float* x, const float* dy, const float* mean, const float* var,
                                  const float* gamma, const float* dgamma, const float* dbeta, float* dx,
                                  uint32_t N, uint32_t C, uint32_t S, float eps, uint64_t limit,
                                  cudaStream_t st, const double* cnt_dev = nullptr);

// ---- layout ops beside the path (k_layout.cu) ----------------------------------
// n = elements (or outputs) the dispatch covers, total = the full index space;
// all index arithmetic is 32-bit (callers refuse index spaces past 2^32).
cudaError_t launch_upsample(const float* x, float* y, uint32_t n, uint32_t total, uint32_t inH, uint32_t inW,
                            uint32_t outH, uint32_t outW, uint32_t sH, uint32_t sW, cudaStream_t st);
cudaError_t launch_upsample_backward(const float* dy, float* dx, uint32_t n, uint32_t total, uint32_t inH,
                                     uint32_t inW, uint32_t outH, uint32_t outW, uint32_t sH, uint32_t sW,
                                     cudaStream_t st);
// rows of L floats: concat writes dst[q*pitch + off + r] = src[q*L + r], slice the reverse
cudaError_t launch_channel_copy(bool slice, const float* src, float* dst, uint32_t n, uint32_t L, uint32_t pitch,
                                uint32_t off, cudaStream_t st);
struct PoolShape {
  uint32_t bc, inH, inW, p, s, outH, outW;     // bc = batch * channels
};
// covered outputs: ow < lw, oh < lh, bc < lb
cudaError_t launch_maxpool_forward(const float* x, float* out, uint32_t* idx, uint32_t lw, uint32_t lh, uint32_t lb,
                                   const PoolShape& g, cudaStream_t st);
cudaError_t launch_maxpool_scatter(const float* dz, const uint32_t* idx, float* d, uint64_t dcount, uint32_t lw,
                                   uint32_t lh, uint32_t lb, uint32_t outH, uint32_t outW, cudaStream_t st);
// the whole dInput (bc*inH*inW floats) in one pass, windows not overlapping
// (s >= p); `flag` is a zeroed device word the call leaves zeroed
cudaError_t launch_maxpool_backward_gather(const float* dz, const uint32_t* idx, float* d, const PoolShape& g,
                                           uint32_t* flag, cudaStream_t st);
// covered: b*P + pixel < lbp, oc < loc
cudaError_t launch_conv_reshape(const float* mm, const float* bias, float* out, uint32_t B, uint32_t OC, uint32_t P,
                                uint32_t lbp, uint32_t loc, uint32_t act, cudaStream_t st);
cudaError_t launch_conv_grad_reshape(const float* dz, const float* fwd, float* out, uint32_t B, uint32_t OC,
                                     uint32_t P, uint32_t lbp, uint32_t loc, cudaStream_t st);

// ---- synthetic data (k_rng.cu) --------------------------------------------------
// Philox4x32-10 counter-based fills.  dist 0: uniform [lo, hi); 1: normal(mean=lo, std=hi)
cudaError_t launch_fill_random(float* y, uint64_t n, uint64_t seed, uint64_t offset, int dist,
                               float lo, float hi, cudaStream_t st);
// x[i] = value for i in the given index list (outlier injection); idx int64
cudaError_t launch_scatter_values(float* x, const int64_t* idx, const float* vals, uint64_t k,
                                  cudaStream_t st);

}  // namespace dct
