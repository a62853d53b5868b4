// Row softmax / log-softmax / cross-entropy kernels of libdct_cuda (sm_100a).
//
// Replaces nn_softmax.hlsl:5-13 (one thread per row, three serial passes),
// nn_loss.hlsl:11-43 (ONE 256-thread group for the whole batch),
// nn_softmax_ce_grad.hlsl:6-11 (re-reads the stored probs) and
// nn_argmax_correct.hlsl:10-26 with ONE fused pass: a warp owns a row, holds
// it in registers (read from HBM once), and writes probs, dlogits =
// (p - onehot) / B and optional log-probs from those registers; each row's
// cross-entropy joins a per-block float64 partial that a second tiny launch
// folds in block order (deterministic).
//
// Accuracy: x - max is formed with an error-free two-sum so the exponent's
// argument is exact to first order (exp(s + t) = exp(s) * (1 + t)); the row
// normaliser is summed in float64, rounded once to its fp32 reciprocal and
// applied as one fp32 product, so each probability carries the error of one
// expf plus two roundings (held to 4 ulp).  The loss and
// log-probs are formed in float64 from log(sum).  dlogits follow the
// reference formula (p - onehot) / B on the rounded p, bit for bit.
#include <algorithm>

#include "dct_common.cuh"
#include "dct_fold.cuh"
#include "dct_tma.cuh"
#include "kernels.h"

namespace dct {

namespace {

constexpr int kSmThreads = 256;
constexpr int kSmWarps = kSmThreads / 32;

// error-free transformation: a + b = s + t exactly (Knuth's TwoSum)
DCT_DEV void two_sum(float a, float b, float& s, float& t) {
  s = __fadd_rn(a, b);
  float bb = __fsub_rn(s, a);
  t = __fadd_rn(__fsub_rn(a, __fsub_rn(s, bb)), __fsub_rn(b, bb));
}

// exp(x - m) with the subtraction carried exactly to first order
DCT_DEV float exp_diff(float x, float m) {
  float s, t;
  two_sum(x, -m, s, t);
  float e = expf(s);
  return __fmaf_rn(e, t, e);
}

DCT_DEV float label_of(const void* labels, bool is_int, uint32_t r, uint32_t K, bool& valid) {
  (void)K;
  if (is_int) {
    int v = reinterpret_cast<const int*>(labels)[r];
    valid = v >= 0;
    return (float)(v < 0 ? 0 : v);
  }
  valid = true;
  return reinterpret_cast<const float*>(labels)[r];
}

// (uint) cast of HLSL: truncation, NaN/negative -> 0, saturate
DCT_DEV uint32_t hlsl_f2u(float f) { return __float2uint_rz(f); }

struct RowCtx {
  const float* __restrict__ logits;
  const void* labels;
  bool labels_int32;
  uint32_t rows, K;
  uint64_t total;          // elements in the logits buffer (label reads stay inside it)
  float* probs;
  float* dlogits;
  float* logprobs;
  double* part;            // per-block fp64 loss partials
  float grad_div;
  bool grad_div_pow2;
  float grad_mul;
  bool ref_max_init;
  bool want_loss;
};

DCT_DEV float grad_of(float p, float oh, const RowCtx& c) {
  const float d = __fsub_rn(p, oh);
  return c.grad_div_pow2 ? __fmul_rn(d, c.grad_mul) : __fdiv_rn(d, c.grad_div);
}

// One warp per row, VPL float4 (VEC) or VPL*4 scalars per lane held in registers.
template <int VPL, bool VEC>
__global__ void __launch_bounds__(kSmThreads) k_softmax_ce_warp(const __grid_constant__ RowCtx c) {
  pdl_entry();
  __shared__ double wsum[kSmWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double block_loss = 0.0;
  const uint32_t K = c.K;
  for (uint32_t r = blockIdx.x * kSmWarps + warp; r < c.rows; r += gridDim.x * kSmWarps) {
    const float* row = c.logits + (uint64_t)r * K;
    float x[VPL * 4];
    // ---- load the row (out-of-range slots = -inf)
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      if (VEC) {
        const uint32_t col = (uint32_t)(lane + 32 * j) * 4;
        float4 v = col < K ? ld_stream4(row + col) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        x[4 * j + 0] = v.x; x[4 * j + 1] = v.y; x[4 * j + 2] = v.z; x[4 * j + 3] = v.w;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t col = (uint32_t)(lane + 32 * (4 * j + q));
          x[4 * j + q] = col < K ? ld_stream(row + col) : -INFINITY;
        }
      }
    }
    // ---- row max
    float m = c.ref_max_init ? -1e30f : -INFINITY;
#pragma unroll
    for (int k = 0; k < VPL * 4; ++k) m = fmaxf(m, x[k]);
    m = warp_max_f(m);
    // ---- exp and float64 normaliser
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < VPL * 4; ++k) {
      const float e = (x[k] == -INFINITY) ? 0.0f : exp_diff(x[k], m);
      s += (double)e;
      x[k] = e;                      // keep e, the logits are no longer needed except for the label
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float invf = (float)(1.0 / s);   // p = e * (1/s): <= 1 ulp on top of exp's
    const double lse = log(s);       // log sum exp(x - m)
    // ---- label
    bool lvalid = true;
    float lab = 0.0f;
    if (c.labels) lab = label_of(c.labels, c.labels_int32, r, K, lvalid);
    const uint32_t lidx = !lvalid ? 0xffffffffu : (c.labels_int32 ? (uint32_t)lab : hlsl_f2u(lab));
    // ---- outputs
    float* prow = c.probs ? c.probs + (uint64_t)r * K : nullptr;
    float* grow = c.dlogits ? c.dlogits + (uint64_t)r * K : nullptr;
    float* lrow = c.logprobs ? c.logprobs + (uint64_t)r * K : nullptr;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      float p[4], g[4];
      uint32_t col0 = VEC ? (uint32_t)(lane + 32 * j) * 4 : 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t col = VEC ? col0 + q : (uint32_t)(lane + 32 * (4 * j + q));
        p[q] = __fmul_rn(x[4 * j + q], invf);
        const float oh = (c.labels && col == lidx) ? 1.0f : 0.0f;
        g[q] = grad_of(p[q], oh, c);
      }
      if (VEC) {
        if (col0 < K) {
          if (prow) st_stream4(prow + col0, make_float4(p[0], p[1], p[2], p[3]));
          if (grow) st_stream4(grow + col0, make_float4(g[0], g[1], g[2], g[3]));
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t col = (uint32_t)(lane + 32 * (4 * j + q));
          if (col < K) {
            if (prow) st_stream(prow + col, p[q]);
            if (grow) st_stream(grow + col, g[q]);
          }
        }
      }
    }
    if (lrow) {
      // log p = (x - m) - lse: re-read the row (L2-resident) and form it in fp64
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t col = VEC ? (uint32_t)(lane + 32 * j) * 4 + q : (uint32_t)(lane + 32 * (4 * j + q));
          if (col < K) lrow[col] = (float)(((double)row[col] - (double)m) - lse);
        }
      }
    }
    if (c.want_loss && lane == 0 && lvalid) {
      const uint64_t li = (uint64_t)r * K + lidx;
      const double xl = li < c.total ? (double)row[lidx] : 0.0;
      block_loss += -((xl - (double)m) - lse);
    }
  }
  if (c.want_loss) {
    if (lane == 0) wsum[warp] = block_loss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int w = 0; w < kSmWarps; ++w) t += wsum[w];
      c.part[blockIdx.x] = t;
    }
  }
}

// TMA-staged variant (K % 4 == 0, row <= 8 KB, no log-probs).  Block b owns the
// WPB * kTmaRows consecutive rows starting at b * WPB * kTmaRows; warp w takes
// rows base + i * WPB + w, i < kTmaRows, so at every step a block's warps cover
// WPB adjacent rows and the grid sweeps the logits in address order (blocks are
// not persistent: the hardware scheduler starts them in index order, as in the
// chunked elementwise schedule).  Each warp owns a two-stage ring of row buffers
// in shared memory filled by 1-D bulk copies (the TMA engine) completing on
// mbarriers: both of its rows are requested up front, so the second streams in
// while the first is computed.  A landed row is read into registers (VPL float4
// per lane) and its stage handed back at once; max, exp with the float64 sum,
// then probabilities and gradients come from registers.  Every mbarrier wait is
// bounded (dct_tma.cuh); a wait that runs out stops the warp's copies and output.
// (The persistent grid-stride form of this kernel reached 0.84 of the copy peak
// on logits[65536, 1000]; this schedule 0.99, at the level of a trivial-compute
// probe of the same one-read, two-write row pattern.)
constexpr int kTmaRows = 2;

template <int VPL, int WPB, bool POW2>
__global__ void __launch_bounds__(WPB * 32) k_softmax_ce_tma(const __grid_constant__ RowCtx c, uint32_t buf_bytes,
                                                             uint32_t* err) {
  pdl_entry();
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ double wsum[WPB];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + 2 * warp;
  float* const buf0 = reinterpret_cast<float*>(smem + 128 + (size_t)(2 * warp) * buf_bytes);
  float* const buf1 = reinterpret_cast<float*>(smem + 128 + (size_t)(2 * warp + 1) * buf_bytes);
  const uint32_t K = c.K;
  const uint32_t rb = K * 4u;
  const uint32_t base = blockIdx.x * (uint32_t)(WPB * kTmaRows) + warp;
  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int s2 = 0; s2 < 2 && s2 < kTmaRows; ++s2) {
      const uint32_t r = base + s2 * WPB;
      if (r < c.rows) {
        mbar_arrive_expect_tx(&bars[s2], rb);
        bulk_load(s2 ? buf1 : buf0, c.logits + (uint64_t)r * K, rb, &bars[s2]);
      }
    }
  }
  __syncwarp();
  double block_loss = 0.0;
#pragma unroll 1
  for (int i = 0; i < kTmaRows; ++i) {
    const uint32_t r = base + i * WPB;
    if (r >= c.rows) break;
    const int st = i & 1;
    float* row = st ? buf1 : buf0;
    bool lvalid = true;
    float lab = 0.0f;
    if (c.labels) lab = label_of(c.labels, c.labels_int32, r, K, lvalid);
    const bool landed = mbar_wait(&bars[st], (uint32_t)(i >> 1) & 1u, err);
    if (__any_sync(0xffffffffu, !landed)) {
      // the row never landed (the error bit is set): issue no more copies, write
      // nothing for this row, and wait (bounded again) for the copies still in
      // flight into this warp's stages before leaving, so none lands in shared
      // memory after the block exits
      mbar_wait(&bars[st], (uint32_t)(i >> 1) & 1u, err);
      if (i + 1 < kTmaRows && r + WPB < c.rows) mbar_wait(&bars[st ^ 1], (uint32_t)((i + 1) >> 1) & 1u, err);
      break;
    }
    const uint32_t lidx = (!lvalid || !c.labels) ? 0xffffffffu : (c.labels_int32 ? (uint32_t)lab : hlsl_f2u(lab));
    float4 x[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint32_t col = (uint32_t)(lane + 32 * j) * 4;
      x[j] = col < K ? *reinterpret_cast<const float4*>(row + col)
                     : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
    // the label's logit (a label >= K reads the flat buffer at r*K + label, as the
    // reference's loss does)
    float xl = 0.0f;
    if (c.want_loss && lvalid) {
      if (lidx < K) {
        xl = row[lidx];
      } else {
        const uint64_t li = (uint64_t)r * K + lidx;
        xl = li < c.total ? c.logits[li] : 0.0f;
      }
    }
    // hand the stage back to the bulk-copy engine for this warp's row i + 2
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && i + 2 < kTmaRows) {
      const uint32_t nr = r + 2 * WPB;
      if (nr < c.rows) {
        mbar_arrive_expect_tx(&bars[st], rb);
        bulk_load(row, c.logits + (uint64_t)nr * K, rb, &bars[st]);
      }
    }
    // row max, and whether any logit is -inf (exp(-inf - m) needs a guard)
    float m = c.ref_max_init ? -1e30f : -INFINITY;
    float mn = INFINITY;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      m = fmaxf(fmaxf(m, fmaxf(x[j].x, x[j].y)), fmaxf(x[j].z, x[j].w));
      const uint32_t col = (uint32_t)(lane + 32 * j) * 4;
      if (col < K) mn = fminf(fminf(mn, fminf(x[j].x, x[j].y)), fminf(x[j].z, x[j].w));
    }
    m = warp_max_f(m);
    const bool ninf = __any_sync(0xffffffffu, mn == -INFINITY);
    // e = exp(x - m), float64 normaliser (padding slots are -inf and give 0)
    double sacc = 0.0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint32_t col = (uint32_t)(lane + 32 * j) * 4;
      if (col < K) {
        float4 v = x[j];
        if (!ninf) {
          v.x = exp_diff(v.x, m);
          v.y = exp_diff(v.y, m);
          v.z = exp_diff(v.z, m);
          v.w = exp_diff(v.w, m);
        } else {
          v.x = (v.x == -INFINITY) ? 0.0f : exp_diff(v.x, m);
          v.y = (v.y == -INFINITY) ? 0.0f : exp_diff(v.y, m);
          v.z = (v.z == -INFINITY) ? 0.0f : exp_diff(v.z, m);
          v.w = (v.w == -INFINITY) ? 0.0f : exp_diff(v.w, m);
        }
        sacc += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
        x[j] = v;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
    const float invf = (float)__drcp_rn(sacc);          // correctly rounded 1/sum, then rounded to float
    // probabilities and gradients (p - onehot) / B: p / B everywhere, the label's
    // one element patched in its float4
    float* prow = c.probs ? c.probs + (uint64_t)r * K : nullptr;
    float* grow = c.dlogits ? c.dlogits + (uint64_t)r * K : nullptr;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint32_t col = (uint32_t)(lane + 32 * j) * 4;
      if (col < K) {
        const float4 e = x[j];
        const float4 p = make_float4(__fmul_rn(e.x, invf), __fmul_rn(e.y, invf), __fmul_rn(e.z, invf),
                                     __fmul_rn(e.w, invf));
        if (prow) st_stream4(prow + col, p);
        if (grow) {
          float4 g;
          if constexpr (POW2) {
            g = make_float4(__fmul_rn(p.x, c.grad_mul), __fmul_rn(p.y, c.grad_mul), __fmul_rn(p.z, c.grad_mul),
                            __fmul_rn(p.w, c.grad_mul));
          } else {
            g = make_float4(__fdiv_rn(p.x, c.grad_div), __fdiv_rn(p.y, c.grad_div), __fdiv_rn(p.z, c.grad_div),
                            __fdiv_rn(p.w, c.grad_div));
          }
          const uint32_t q = lidx - col;                  // the label falls in this float4
          if (q < 4u) {
            if (q == 0) g.x = grad_of(p.x, 1.0f, c);
            else if (q == 1) g.y = grad_of(p.y, 1.0f, c);
            else if (q == 2) g.z = grad_of(p.z, 1.0f, c);
            else g.w = grad_of(p.w, 1.0f, c);
          }
          st_stream4(grow + col, g);
        }
      }
    }
    if (c.want_loss && lane == 0 && lvalid) {
      // float log of the row sum: about 1 ulp of log(sum), far below the loss's rel 1e-5
      block_loss += -(((double)xl - (double)m) - (double)logf((float)sacc));
    }
  }
  if (c.want_loss) {
    if (lane == 0) wsum[warp] = block_loss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int w = 0; w < WPB; ++w) t += wsum[w];
      c.part[blockIdx.x] = t;
    }
  }
}

// Rows longer than 2048: one block per row, three streaming passes (L2 keeps the row).
__global__ void __launch_bounds__(kSmThreads) k_softmax_ce_block(const __grid_constant__ RowCtx c) {
  pdl_entry();
  __shared__ double shd[32];
  __shared__ float shf[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double block_loss = 0.0;
  const uint32_t K = c.K;
  for (uint32_t r = blockIdx.x; r < c.rows; r += gridDim.x) {
    const float* row = c.logits + (uint64_t)r * K;
    float m = c.ref_max_init ? -1e30f : -INFINITY;
    for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, row[k]);
    m = warp_max_f(m);
    __syncthreads();
    if (lane == 0) shf[warp] = m;
    __syncthreads();
    m = shf[0];
    for (int w = 1; w < kSmWarps; ++w) m = fmaxf(m, shf[w]);
    double s = 0.0;
    for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) {
      const float xv = row[k];
      s += (xv == -INFINITY) ? 0.0 : (double)exp_diff(xv, m);
    }
    s = block_sum(s, shd);
    __syncthreads();
    if (threadIdx.x == 0) shd[0] = s;
    __syncthreads();
    s = shd[0];
    const float invf = (float)(1.0 / s);
    const double lse = log(s);
    bool lvalid = true;
    float lab = 0.0f;
    if (c.labels) lab = label_of(c.labels, c.labels_int32, r, K, lvalid);
    const uint32_t lidx = !lvalid ? 0xffffffffu : (c.labels_int32 ? (uint32_t)lab : hlsl_f2u(lab));
    for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) {
      const float xv = row[k];
      const float e = (xv == -INFINITY) ? 0.0f : exp_diff(xv, m);
      const float p = __fmul_rn(e, invf);
      if (c.probs) c.probs[(uint64_t)r * K + k] = p;
      if (c.dlogits) c.dlogits[(uint64_t)r * K + k] = grad_of(p, (c.labels && k == lidx) ? 1.0f : 0.0f, c);
      if (c.logprobs) c.logprobs[(uint64_t)r * K + k] = (float)(((double)xv - (double)m) - lse);
    }
    if (c.want_loss && threadIdx.x == 0 && lvalid) {
      const uint64_t li = (uint64_t)r * K + lidx;
      const double xl = li < c.total ? (double)row[lidx] : 0.0;
      block_loss += -((xl - (double)m) - lse);
    }
    __syncthreads();
  }
  if (c.want_loss && threadIdx.x == 0) c.part[blockIdx.x] = block_loss;
}

__global__ void k_loss_final(const double* part, int nparts, double div, float* loss, double* raw) {
  pdl_entry();
  __shared__ double sh[32];
  const double acc = strided_sum(part, nparts);
  double t = block_sum(acc, sh);
  if (threadIdx.x == 0) {
    if (raw) raw[0] = t;
    if (loss) loss[0] = (float)(t / div);
  }
}

// The same fold for a sharded batch, in the same launch as the exchange over
// peer memory: thread 0 stores this rank's loss sum (record word 0) into every
// peer's slot, block 0 the header [rows, valid, -], and thread 0 folds every
// rank's record in rank order into loss = sum / div (fold_loss).
__global__ void k_loss_final_xchg(const double* part, int nparts, double div, float* loss,
                                  const __grid_constant__ PeerXfer p) {
  pdl_entry();
  __shared__ double sh[32];
  bool gave_up = false;
  peer_put_header(p);
  const double acc = strided_sum(part, nparts);
  const double t = block_sum(acc, sh);
  if (threadIdx.x == 0) {
    peer_put_word(p, 0, (unsigned long long)__double_as_longlong(t));
    fold_loss(PeerRecsOwn0{p, gave_up, t}, p.world, div, loss, p.err);
  }
  peer_sync(p, gave_up);
}

int softmax_blocks(uint32_t rows, uint32_t K) {
  const DevInfo& d = dev_info();
  if (K > 2048) {
    int b = d.sm_count * 8;
    return (int)(rows < (uint32_t)b ? (rows ? rows : 1) : b);
  }
  uint64_t need = ((uint64_t)rows + kSmWarps - 1) / kSmWarps;
  uint64_t cap = (uint64_t)d.sm_count * 16;
  uint64_t b = need < cap ? need : cap;
  return (int)(b ? b : 1);
}

}  // namespace

// Shared-memory stage of one row (16-byte multiple, the bulk copy's rule) and
// warps per block of the TMA-staged kernel.  For rows up to 1024 floats, 7
// warps per block let 4 blocks (28 warps) fit an SM's 228 KB with two stages
// per warp; 8 warps fit only 3 blocks (24 warps).
static uint32_t tma_stage_bytes(uint32_t K) { return ((K * 4u) + 15u) & ~15u; }
static int tma_warps(uint32_t K) { return tma_stage_bytes(K) <= 4096 ? 7 : 4; }

// The block-order fold of the per-block loss partials: loss / loss_partial,
// or, for a sharded batch over peer memory, the exchange and the rank fold.
static cudaError_t launch_loss_fold(const RowCtx& c, int nparts, const SoftmaxCEArgs& a, cudaStream_t st) {
  if (a.xchg) launch_pdl(k_loss_final_xchg, dim3(1), dim3(1024), 0, st, c.part, nparts, a.loss_div, a.loss, *a.xchg);
  else launch_pdl(k_loss_final, dim3(1), dim3(1024), 0, st, c.part, nparts, a.loss_div, a.loss, a.loss_partial);
  return cudaGetLastError();
}

// blocks of the TMA-staged kernel: one per WPB * kTmaRows consecutive rows
int tma_blocks(uint32_t rows, uint32_t K) {
  const uint64_t per = (uint64_t)tma_warps(K) * kTmaRows;
  return (int)std::max<uint64_t>(1, ((uint64_t)rows + per - 1) / per);
}

size_t softmax_ce_ws_bytes(uint32_t rows, uint32_t K) {
  return (size_t)std::max(softmax_blocks(rows, K), tma_blocks(rows, K)) * sizeof(double) + 64;
}

cudaError_t launch_softmax_ce(const SoftmaxCEArgs& a, void* ws, cudaStream_t st) {
  if (a.rows == 0) {
    // the loss is the empty sum over its divisor: 0, or NaN (0 / 0) when the
    // divisor is the empty batch itself, as nn_loss.hlsl:41 computes it
    if (a.loss) {
      cudaError_t e = cudaMemsetAsync(a.loss, a.loss_div != 0.0 ? 0 : 0xFF, sizeof(float), st);
      if (e) return e;
    }
    if (a.loss_partial) return cudaMemsetAsync(a.loss_partial, 0, sizeof(double), st);
    return cudaSuccess;
  }
  if (a.K == 0) return cudaErrorInvalidValue;
  RowCtx c;
  c.logits = a.logits;
  c.labels = a.labels;
  c.labels_int32 = a.labels_int32;
  c.rows = a.rows;
  c.K = a.K;
  c.total = (uint64_t)a.rows * a.K;
  c.probs = a.probs;
  c.dlogits = a.dlogits;
  c.logprobs = a.logprobs;
  c.want_loss = (a.loss != nullptr || a.loss_partial != nullptr || a.xchg != nullptr) && a.labels != nullptr;
  c.part = (double*)ws;
  if (c.want_loss && !ws) return cudaErrorInvalidValue;
  c.grad_div = a.grad_div;
  int ex = 0;
  const float fr = frexpf(a.grad_div, &ex);
  c.grad_div_pow2 = (fr == 0.5f) && a.grad_div > 0.0f && ex - 1 > -126 && ex - 1 < 127;
  c.grad_mul = c.grad_div_pow2 ? ldexpf(1.0f, -(ex - 1)) : 1.0f;
  c.ref_max_init = a.ref_max_init;
  if (a.dlogits && !a.labels) return cudaErrorInvalidValue;
  const bool vec = (a.K % 4 == 0) && aligned16_h(a.logits) && (!a.probs || aligned16_h(a.probs)) &&
                   (!a.dlogits || aligned16_h(a.dlogits));
  const uint32_t K = a.K;
  if (vec && !a.logprobs && K <= 2048 && K >= 128) {
    const uint32_t buf_bytes = tma_stage_bytes(K);
    const int wpb = tma_warps(K);
    const size_t smem = 128 + (size_t)2 * wpb * buf_bytes;
    const int blocks_t = tma_blocks(a.rows, K);
    cudaError_t e = cudaSuccess;
#define DCT_SM_TMA2(VPL, WPB, P2)                                                                             \
  do {                                                                                                        \
    static bool attr_set = false;                                                                             \
    if (!attr_set) {                                                                                          \
      e = cudaFuncSetAttribute(k_softmax_ce_tma<VPL, WPB, P2>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                               (int)(128 + 2 * WPB * 8192));                                                   \
      attr_set = (e == cudaSuccess);                                                                          \
    }                                                                                                         \
    if (e == cudaSuccess) launch_pdl(k_softmax_ce_tma<VPL, WPB, P2>, dim3(blocks_t), dim3(WPB * 32), smem, st, c, buf_bytes, a.err); \
  } while (0)
#define DCT_SM_TMA(VPL, WPB)                                                                                  \
  do {                                                                                                        \
    if (c.grad_div_pow2) DCT_SM_TMA2(VPL, WPB, true);                                                         \
    else DCT_SM_TMA2(VPL, WPB, false);                                                                        \
  } while (0)
    if (K <= 256) DCT_SM_TMA(2, 7);
    else if (K <= 512) DCT_SM_TMA(4, 7);
    else if (K <= 1024) DCT_SM_TMA(8, 7);
    else DCT_SM_TMA(16, 4);
#undef DCT_SM_TMA
#undef DCT_SM_TMA2
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess || !c.want_loss) return e;
    return launch_loss_fold(c, blocks_t, a, st);
  }
  const int blocks = softmax_blocks(a.rows, a.K);
  if (K <= 128) {
    if (vec) launch_pdl(k_softmax_ce_warp<1, true>, dim3(blocks), dim3(kSmThreads), 0, st, c);
    else launch_pdl(k_softmax_ce_warp<1, false>, dim3(blocks), dim3(kSmThreads), 0, st, c);
  } else if (K <= 256) {
    if (vec) launch_pdl(k_softmax_ce_warp<2, true>, dim3(blocks), dim3(kSmThreads), 0, st, c);
    else launch_pdl(k_softmax_ce_warp<2, false>, dim3(blocks), dim3(kSmThreads), 0, st, c);
  } else if (K <= 512) {
    if (vec) launch_pdl(k_softmax_ce_warp<4, true>, dim3(blocks), dim3(kSmThreads), 0, st, c);
    else launch_pdl(k_softmax_ce_warp<4, false>, dim3(blocks), dim3(kSmThreads), 0, st, c);
  } else if (K <= 1024) {
    if (vec) launch_pdl(k_softmax_ce_warp<8, true>, dim3(blocks), dim3(kSmThreads), 0, st, c);
    else launch_pdl(k_softmax_ce_warp<8, false>, dim3(blocks), dim3(kSmThreads), 0, st, c);
  } else if (K <= 2048) {
    if (vec) launch_pdl(k_softmax_ce_warp<16, true>, dim3(blocks), dim3(kSmThreads), 0, st, c);
    else launch_pdl(k_softmax_ce_warp<16, false>, dim3(blocks), dim3(kSmThreads), 0, st, c);
  } else {
    launch_pdl(k_softmax_ce_block, dim3(blocks), dim3(kSmThreads), 0, st, c);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !c.want_loss) return e;
  return launch_loss_fold(c, blocks, a, st);
}

// ---------------------------------------------------------------------------
// reference argmax_correct (nn_argmax_correct.hlsl:10-26): strict '>' scan
// from column 0; equivalent parallel rule: a NaN at column 0 gives index 0,
// other NaNs are never chosen, ties keep the lowest index.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_argmax_correct(const float* __restrict__ logits,
                                                        const float* __restrict__ labels, uint32_t rows, uint32_t K,
                                                        uint32_t* counter) {
  pdl_entry();
  __shared__ uint32_t sc[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t hits = 0;
  for (uint32_t r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
    const float* row = logits + (uint64_t)r * K;
    float bv = 0.0f;
    int64_t bi = -1;
    for (uint32_t k = lane; k < K; k += 32) {
      const float v = row[k];
      if (isnan(v)) continue;
      if (bi < 0 || v > bv) { bv = v; bi = k; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
      const uint32_t idx = isnan(row[0]) ? 0u : (bi < 0 ? 0u : (uint32_t)bi);
      if (idx == hlsl_f2u(labels[r])) ++hits;
    }
  }
  if (lane == 0) sc[warp] = hits;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < 8; ++w) t += sc[w];
    if (t) atomicAdd(counter, t);
  }
}

cudaError_t launch_argmax_correct(const float* logits, const float* labels, uint32_t rows, uint32_t K,
                                  uint32_t* counter, cudaStream_t st) {
  if (rows == 0 || K == 0) return cudaSuccess;
  const DevInfo& d = dev_info();
  uint32_t blocks = (rows + 7) / 8;
  const uint32_t cap = (uint32_t)d.sm_count * 8;
  if (blocks > cap) blocks = cap;
  launch_pdl(k_argmax_correct, dim3(blocks), dim3(256), 0, st, logits, labels, rows, K, counter);
  return cudaGetLastError();
}

}  // namespace dct
