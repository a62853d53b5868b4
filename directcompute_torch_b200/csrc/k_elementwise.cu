// Elementwise and broadcast kernels of libdct_cuda (sm_100a).
//
// Replaces the reference's one-thread-per-element HLSL shaders
// (nn_add_bias.hlsl, nn_bias_relu.hlsl, nn_relu*.hlsl, nn_leaky_relu*.hlsl,
// nn_sigmoid*.hlsl, nn_add.hlsl, nn_scale_add.hlsl, nn_grad_accum.hlsl,
// nn_global_avg_pool_backward.hlsl, nn_softmax_ce_grad.hlsl,
// nn_accumulate_scalar.hlsl, nn_dice_loss_grad.hlsl) and adds the N-d
// NumPy-broadcast binary ops and exp/log/tanh the reference only has on its
// NumPy side.
//
// Design: 128-bit vectors with streaming cache hints over a chunked block
// schedule (see "Schedule" below); broadcast operands are resolved from the
// output index with Granlund-Montgomery fast division over the collapsed
// dims, and small broadcast rows are served from L1.  All arithmetic uses the
// round-to-nearest intrinsics so no multiply-add is ever contracted: the
// results are bit-identical to the fp32 formulas of the shaders / NumPy.
#include <algorithm>

#include "dct_common.cuh"
#include "dct_math.cuh"
#include "kernels.h"

namespace dct {

// ---------------------------------------------------------------------------
// scalar op definitions
// ---------------------------------------------------------------------------
template <int OP>
DCT_DEV float unary_op(float x, float alpha) {
  if constexpr (OP == EW_RELU) {
    return x > 0.0f ? x : 0.0f;                       // HLSL max(0,x): NaN -> 0
  } else if constexpr (OP == EW_RELU6) {
    return x > 0.0f ? (x < 6.0f ? x : 6.0f) : 0.0f;
  } else if constexpr (OP == EW_LEAKY_RELU) {
    return x > 0.0f ? x : __fmul_rn(x, alpha);
  } else if constexpr (OP == EW_SIGMOID) {
    return sigmoid_acc(x);                            // <= 1.5 ulp, branch-free (dct_math.cuh)
  } else if constexpr (OP == EW_EXP) {
    return expf(x);
  } else if constexpr (OP == EW_LOG_ABS1P) {
    return logf(__fadd_rn(fabsf(x), 1.0f));           // NumPy: log(float32(|x| + 1))
  } else if constexpr (OP == EW_TANH) {
    return tanhf(x);
  } else if constexpr (OP == EW_NEG) {
    return -x;
  } else {
    return fabsf(x);
  }
}

template <int OP>
DCT_DEV float binary_op(float a, float b, float alpha, float beta) {
  if constexpr (OP == EW_ADD) {
    return __fadd_rn(a, b);
  } else if constexpr (OP == EW_SUB) {
    return __fsub_rn(a, b);
  } else if constexpr (OP == EW_MUL) {
    return __fmul_rn(a, b);
  } else if constexpr (OP == EW_DIV) {
    return __fdiv_rn(a, b);
  } else if constexpr (OP == EW_MAXIMUM) {
    return (a > b || isnan(a)) ? a : b;                // np.maximum incl. NaN / signed zeros
  } else if constexpr (OP == EW_MINIMUM) {
    return (a < b || isnan(a)) ? a : b;
  } else if constexpr (OP == EW_RELU_GRAD) {           // (grad, x)
    return b > 0.0f ? a : 0.0f;
  } else if constexpr (OP == EW_RELU6_GRAD) {
    return (b > 0.0f && b < 6.0f) ? a : 0.0f;
  } else if constexpr (OP == EW_LEAKY_RELU_GRAD) {
    return __fmul_rn(a, b > 0.0f ? 1.0f : alpha);
  } else if constexpr (OP == EW_SIGMOID_GRAD) {        // (dy, y): dy*y*(1-y)
    return __fmul_rn(__fmul_rn(a, b), __fsub_rn(1.0f, b));
  } else if constexpr (OP == EW_PICK_MAX) {            // maximum's gradient goes to a
    return (a >= b || isnan(a)) ? 1.0f : 0.0f;
  } else if constexpr (OP == EW_PICK_MIN) {
    return (a <= b || isnan(a)) ? 1.0f : 0.0f;
  } else if constexpr (OP == EW_EXP_GRAD) {            // (g, y = exp(x)): g*y
    return __fmul_rn(a, b);
  } else if constexpr (OP == EW_TANH_GRAD) {           // (g, y = tanh(x)): g*(1-y*y)
    return __fmul_rn(a, __fsub_rn(1.0f, __fmul_rn(b, b)));
  } else if constexpr (OP == EW_LOG_ABS1P_GRAD) {      // (g, x): g*sign(x)/(|x|+1)
    const float q = __fdiv_rn(a, __fadd_rn(fabsf(b), 1.0f));
    return b > 0.0f ? q : (b < 0.0f ? -q : (b == 0.0f ? 0.0f : b));
  } else if constexpr (OP == EW_FIRST) {               // broadcast copy of a
    return a;
  } else {                                             // EW_SCALE_ADD
    return __fadd_rn(__fmul_rn(alpha, a), __fmul_rn(beta, b));
  }
}

template <int OP>
DCT_DEV float4 unary4(float4 v, float al) {
  return make_float4(unary_op<OP>(v.x, al), unary_op<OP>(v.y, al), unary_op<OP>(v.z, al),
                     unary_op<OP>(v.w, al));
}
template <int OP>
DCT_DEV float4 binary4(float4 a, float4 b, float al, float be) {
  return make_float4(binary_op<OP>(a.x, b.x, al, be), binary_op<OP>(a.y, b.y, al, be),
                     binary_op<OP>(a.z, b.z, al, be), binary_op<OP>(a.w, b.w, al, be));
}

// ---------------------------------------------------------------------------
// Schedule.  Streaming kernels use CHUNKED blocks: block b owns the contiguous
// output range [b*kChunk4, (b+1)*kChunk4) of float4s (16 KB), its 256 threads
// hold kChunkU vectors each with every load issued before any store, and the
// grid has one block per chunk, so the hardware block scheduler sweeps memory
// in address order.  On B200 this keeps the set of open DRAM pages small: a
// copy stream measured 6.5-6.9 TB/s this way against 5.9-6.2 TB/s for a
// grid-stride loop over the same bytes (and 6.5 TB/s for torch's copy_).
// Unaligned or >2^40-element inputs fall back to scalar grid-stride loops.
// Inputs may alias the output (in-place grad_accum / Muon's scale_add): every
// element is read and written by one thread, loads first.
// ---------------------------------------------------------------------------
constexpr int kChunkU = 4;
constexpr uint64_t kChunk4 = 256ull * kChunkU;

inline unsigned chunk_blocks(uint64_t n4) { return (unsigned)((n4 + kChunk4 - 1) / kChunk4); }

template <int OP>
__global__ void __launch_bounds__(256) k_unary_chunk(const float* x, float* y, uint64_t n, float al) {
  pdl_entry();
  const uint64_t n4 = n >> 2;
  const uint64_t base = (uint64_t)blockIdx.x * kChunk4 + threadIdx.x;
  float4 v[kChunkU];
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) v[k] = ld_stream4(x + 4 * i);
  }
  if constexpr (OP == EW_SIGMOID) {
    // the sigmoid's 2^(j/32) table in shared memory, one private copy per warp
    // (a warp-level sync, no block barrier): one 8-byte load per element
    __shared__ float2 tabs[8][32];
    float2* tab = tabs[threadIdx.x >> 5];
    tab[threadIdx.x & 31] = kExp2Tab[threadIdx.x & 31];
    __syncwarp();
#pragma unroll
    for (int k = 0; k < kChunkU; ++k) {
      const uint64_t i = base + 256ull * k;
      if (i < n4)
        st_stream4(y + 4 * i, make_float4(sigmoid_tab(v[k].x, tab), sigmoid_tab(v[k].y, tab),
                                          sigmoid_tab(v[k].z, tab), sigmoid_tab(v[k].w, tab)));
    }
  } else {
#pragma unroll
    for (int k = 0; k < kChunkU; ++k) {
      const uint64_t i = base + 256ull * k;
      if (i < n4) st_stream4(y + 4 * i, unary4<OP>(v[k], al));
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const uint64_t t = 4 * n4 + threadIdx.x;
    y[t] = unary_op<OP>(x[t], al);
  }
}

template <int OP>
__global__ void __launch_bounds__(256) k_unary_scalar(const float* x, float* y, uint64_t n, float al) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = unary_op<OP>(x[i], al);
}

template <int OP>
__global__ void __launch_bounds__(256) k_binary_chunk(const float* a, const float* b, float* y, uint64_t n,
                                                      float al, float be) {
  pdl_entry();
  const uint64_t n4 = n >> 2;
  const uint64_t base = (uint64_t)blockIdx.x * kChunk4 + threadIdx.x;
  float4 va[kChunkU], vb[kChunkU];
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) { va[k] = ld_stream4(a + 4 * i); vb[k] = ld_stream4(b + 4 * i); }
  }
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) st_stream4(y + 4 * i, binary4<OP>(va[k], vb[k], al, be));
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const uint64_t t = 4 * n4 + threadIdx.x;
    y[t] = binary_op<OP>(a[t], b[t], al, be);
  }
}

template <int OP>
__global__ void __launch_bounds__(256) k_binary_scalar(const float* a, const float* b, float* y,
                                                       uint64_t n, float al, float be) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = binary_op<OP>(a[i], b[i], al, be);
}

// ---------------------------------------------------------------------------
// broadcast kernels.  The output is viewed as ROWS x Q (Q = innermost
// collapsed dim, contiguous in the output).  Each operand has a per-row base
// offset (from the outer multi-index) and an inner stride of 1 or 0.
// ---------------------------------------------------------------------------
constexpr int kMaxDims = 8;

struct RowMap {
  int nouter;                       // outer (row) dims, <= kMaxDims - 1
  FastDiv q4div;                    // float4s per output row
  FastDiv div[kMaxDims];            // outer extents, innermost outer dim first
  int64_t a_str[kMaxDims];          // per outer dim, same order
  int64_t b_str[kMaxDims];
};

DCT_DEV void row_offsets(const RowMap& m, uint32_t row, int64_t& ao, int64_t& bo) {
  ao = 0;
  bo = 0;
  for (int d = 0; d < m.nouter; ++d) {
    uint32_t q = m.div[d].div(row);
    uint32_t r = row - q * m.div[d].d;
    ao += (int64_t)r * m.a_str[d];
    bo += (int64_t)r * m.b_str[d];
    row = q;
  }
}

// General broadcast, vector path: Q % 4 == 0 and every contiguous operand row
// 16-byte aligned.  A_BC / B_BC: operand broadcast along the inner dim
// (a scalar per row, replicated in registers).  Output float4 index i
// (< 2^32) -> row = i / q4, c4 = i - row*q4 -> operand row offsets.
template <int OP, bool A_BC, bool B_BC>
DCT_DEV float4 bcast_val(const float* __restrict__ a, const float* __restrict__ b, const RowMap& m, uint32_t i) {
  const uint32_t row = m.q4div.div(i);
  const uint32_t c4 = i - row * m.q4div.d;
  int64_t ao, bo;
  row_offsets(m, row, ao, bo);
  float4 va, vb;
  if (A_BC) { float s = ld_keep(a + ao); va = make_float4(s, s, s, s); }
  else va = ld_keep4(a + ao + 4 * (int64_t)c4);
  if (B_BC) { float s = ld_keep(b + bo); vb = make_float4(s, s, s, s); }
  else vb = ld_keep4(b + bo + 4 * (int64_t)c4);
  return binary4<OP>(va, vb, 0.f, 0.f);
}

template <int OP, bool A_BC, bool B_BC>
__global__ void __launch_bounds__(256) k_bcast_chunk(const float* __restrict__ a, const float* __restrict__ b,
                                                     float* __restrict__ y, uint32_t n4,
                                                     const __grid_constant__ RowMap m) {
  pdl_entry();
  const uint64_t base = (uint64_t)blockIdx.x * kChunk4 + threadIdx.x;
  float4 o[kChunkU];
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) o[k] = bcast_val<OP, A_BC, B_BC>(a, b, m, (uint32_t)i);
  }
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) st_stream4(y + 4 * i, o[k]);
  }
}

// Three collapsed dims [P, R, Q], both operands contiguous along Q, operand A
// (or B when SWAP) constant along R: y[p, r, q] = op(A[p*sap + q], B[p*sbp + r*sbr + q]).
// Block (q-slice, r-chunk, p): each thread keeps its A float4 in a register
// for the whole r-chunk and streams B (usually L2-resident: the broadcast
// operands are small) into y.  Blocks are numbered q-slice fastest, so the
// blocks of one r-chunk write whole output rows together.
template <int OP, bool SWAP>
__global__ void __launch_bounds__(256) k_bcast3(const float* __restrict__ a, const float* __restrict__ b,
                                                float* __restrict__ y, uint32_t R, uint32_t q4, uint32_t rchunk,
                                                int64_t sap, int64_t sbp, int64_t sbr) {
  pdl_entry();
  const uint32_t c4 = blockIdx.x * 256 + threadIdx.x;
  if (c4 >= q4) return;
  const uint32_t p = blockIdx.z;
  const uint32_t r0 = blockIdx.y * rchunk;
  const uint32_t r1 = min(R, r0 + rchunk);
  const float4 va = ld_keep4(a + (int64_t)p * sap + 4 * (int64_t)c4);
  const float* bp = b + (int64_t)p * sbp + 4 * (int64_t)c4;
  float* yp = y + ((uint64_t)p * R) * (4ull * q4) + 4ull * c4;
  uint32_t r = r0;
  for (; r + 3 < r1; r += 4) {
    float4 vb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) vb[k] = ld_keep4(bp + (int64_t)(r + k) * sbr);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      st_stream4(yp + (uint64_t)(r + k) * (4ull * q4), SWAP ? binary4<OP>(vb[k], va, 0.f, 0.f) : binary4<OP>(va, vb[k], 0.f, 0.f));
  }
  for (; r < r1; ++r) {
    const float4 vb = ld_keep4(bp + (int64_t)r * sbr);
    st_stream4(yp + (uint64_t)r * (4ull * q4), SWAP ? binary4<OP>(vb, va, 0.f, 0.f) : binary4<OP>(va, vb, 0.f, 0.f));
  }
}

// Row broadcast y[r, c] = op(A[r, c], v[c]) (or op(v[c], A[r, c]) when SWAP),
// N % 4 == 0: A streams, the broadcast row is read through L1 (it is at most
// a few hundred KB and every block re-reads the same columns).
template <int OP, bool SWAP, bool RELU>
__global__ void __launch_bounds__(256) k_rowvec_chunk(const float* A, const float* v, float* y, uint32_t n4,
                                                      FastDiv ncol4) {
  pdl_entry();
  const uint64_t base = (uint64_t)blockIdx.x * kChunk4 + threadIdx.x;
  float4 x[kChunkU], bv[kChunkU];
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      const uint32_t ii = (uint32_t)i;
      const uint32_t c4 = ii - ncol4.div(ii) * ncol4.d;
      x[k] = ld_stream4(A + 4 * i);
      bv[k] = ld_keep4(v + 4ull * c4);
    }
  }
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      float4 o = SWAP ? binary4<OP>(bv[k], x[k], 0.f, 0.f) : binary4<OP>(x[k], bv[k], 0.f, 0.f);
      if (RELU) o = unary4<EW_RELU>(o, 0.f);
      st_stream4(y + 4 * i, o);
    }
  }
}

// Scalar fallback for any shape: per element index decomposition.
struct ElemMap {
  int ndim;
  FastDiv div[kMaxDims];            // innermost first
  int64_t a_str[kMaxDims];
  int64_t b_str[kMaxDims];
};

template <int OP>
__global__ void __launch_bounds__(256) k_bcast_scalar(const float* a, const float* b, float* y, uint64_t n,
                                                      const __grid_constant__ ElemMap m) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t rem = (uint32_t)i;
    int64_t ao = 0, bo = 0;
    for (int d = 0; d < m.ndim; ++d) {
      uint32_t q = m.div[d].div(rem);
      uint32_t r = rem - q * m.div[d].d;
      ao += (int64_t)r * m.a_str[d];
      bo += (int64_t)r * m.b_str[d];
      rem = q;
    }
    y[i] = binary_op<OP>(a[ao], b[bo], 0.f, 0.f);
  }
}

// Reference add_bias / bias_relu for N not a multiple of 4: C[i] = A[i] + B[i % N].
template <bool RELU>
__global__ void __launch_bounds__(256) k_add_bias_scalar(const float* A, const float* B, float* C, uint64_t n,
                                                         uint32_t N, FastDiv dn) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t col;
    if (i < 0xffffffffull) { uint32_t ii = (uint32_t)i; col = ii - dn.div(ii) * N; }
    else col = (uint32_t)(i % N);
    float o = __fadd_rn(A[i], ld_keep(B + col));
    C[i] = RELU ? (o > 0.0f ? o : 0.0f) : o;
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
#define DCT_UNARY_CASES(X) X(EW_RELU) X(EW_RELU6) X(EW_LEAKY_RELU) X(EW_SIGMOID) X(EW_EXP) \
  X(EW_LOG_ABS1P) X(EW_TANH) X(EW_NEG) X(EW_ABS)
#define DCT_BINARY_CASES(X) X(EW_ADD) X(EW_SUB) X(EW_MUL) X(EW_DIV) X(EW_MAXIMUM) X(EW_MINIMUM) \
  X(EW_RELU_GRAD) X(EW_RELU6_GRAD) X(EW_LEAKY_RELU_GRAD) X(EW_SIGMOID_GRAD) X(EW_SCALE_ADD)     \
  X(EW_PICK_MAX) X(EW_PICK_MIN) X(EW_EXP_GRAD) X(EW_TANH_GRAD) X(EW_LOG_ABS1P_GRAD) X(EW_FIRST)
#define DCT_BCAST_CASES(X) X(EW_ADD) X(EW_SUB) X(EW_MUL) X(EW_DIV) X(EW_MAXIMUM) X(EW_MINIMUM) \
  X(EW_PICK_MAX) X(EW_PICK_MIN) X(EW_FIRST)

constexpr uint64_t kMaxChunkN4 = (1ull << 31) * kChunk4;   // grid.x limit

cudaError_t launch_unary(int op, const float* x, float* y, uint64_t n, float alpha, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const bool vec = aligned16_h(x) && aligned16_h(y) && (n >> 2) < kMaxChunkN4;
  const unsigned blocks = vec ? std::max(1u, chunk_blocks(n >> 2)) : grid_for(n, 256);
  switch (op) {
#define X(OPC)                                                                      \
  case OPC:                                                                         \
    if (vec) launch_pdl(k_unary_chunk<OPC>, dim3(blocks), dim3(256), 0, st, x, y, n, alpha);           \
    else launch_pdl(k_unary_scalar<OPC>, dim3(blocks), dim3(256), 0, st, x, y, n, alpha);              \
    break;
    DCT_UNARY_CASES(X)
#undef X
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_binary_same(int op, const float* a, const float* b, float* y, uint64_t n,
                               float alpha, float beta, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const bool vec = aligned16_h(a) && aligned16_h(b) && aligned16_h(y) && (n >> 2) < kMaxChunkN4;
  const unsigned blocks = vec ? std::max(1u, chunk_blocks(n >> 2)) : grid_for(n, 256);
  switch (op) {
#define X(OPC)                                                                        \
  case OPC:                                                                           \
    if (vec) launch_pdl(k_binary_chunk<OPC>, dim3(blocks), dim3(256), 0, st, a, b, y, n, alpha, beta);   \
    else launch_pdl(k_binary_scalar<OPC>, dim3(blocks), dim3(256), 0, st, a, b, y, n, alpha, beta);      \
    break;
    DCT_BINARY_CASES(X)
#undef X
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_add_bias(const float* A, const float* B, float* C, uint64_t M, uint64_t N, bool relu,
                            cudaStream_t st) {
  const uint64_t n = M * N;
  if (n == 0) return cudaSuccess;
  if (N % 4 == 0 && n / 4 < 0xffffffffull && aligned16_h(A) && aligned16_h(B) && aligned16_h(C)) {
    const uint32_t n4 = (uint32_t)(n / 4);
    FastDiv nc((uint32_t)(N / 4));
    if (relu) launch_pdl(k_rowvec_chunk<EW_ADD, false, true>, dim3(chunk_blocks(n4)), dim3(256), 0, st, A, B, C, n4, nc);
    else launch_pdl(k_rowvec_chunk<EW_ADD, false, false>, dim3(chunk_blocks(n4)), dim3(256), 0, st, A, B, C, n4, nc);
  } else {
    if (N == 0 || N > 0xffffffffull) return cudaErrorInvalidValue;
    const unsigned blocks = grid_for(n, 256);
    FastDiv dn((uint32_t)N);
    if (relu) launch_pdl(k_add_bias_scalar<true>, dim3(blocks), dim3(256), 0, st, A, B, C, n, (uint32_t)N, dn);
    else launch_pdl(k_add_bias_scalar<false>, dim3(blocks), dim3(256), 0, st, A, B, C, n, (uint32_t)N, dn);
  }
  return cudaGetLastError();
}

// Collapse adjacent output dims whose operand strides compose (both operands
// contiguous-with-broadcast), then pick the row-vector kernel, the general
// vector kernel, or the scalar fallback.
cudaError_t launch_binary_bcast(int op, const float* a, const float* b, float* y, int ndim,
                                const int64_t* shape, const int64_t* a_str, const int64_t* b_str,
                                cudaStream_t st) {
  if (ndim < 0 || ndim > kMaxDims) return cudaErrorInvalidValue;
  int64_t sh[kMaxDims], as[kMaxDims], bs_[kMaxDims];
  int k = 0;
  uint64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] == 0) return cudaSuccess;
    n *= (uint64_t)shape[d];
    if (shape[d] == 1) continue;                    // size-1 dims carry nothing
    if (k > 0 && as[k - 1] == a_str[d] * shape[d] && bs_[k - 1] == b_str[d] * shape[d]) {
      sh[k - 1] *= shape[d];                        // merge into previous dim
      as[k - 1] = a_str[d];
      bs_[k - 1] = b_str[d];
      continue;
    }
    sh[k] = shape[d]; as[k] = a_str[d]; bs_[k] = b_str[d]; ++k;
  }
  if (k == 0) { sh[0] = 1; as[0] = 0; bs_[0] = 0; k = 1; }
  // Plain same-shape (or fully contiguous) case.
  if (k == 1 && as[0] == 1 && bs_[0] == 1) return launch_binary_same(op, a, b, y, n, 0.f, 0.f, st);
  for (int d = 0; d < k; ++d)
    if (sh[d] > 0xffffffffll) return cudaErrorInvalidValue;

  const int64_t Q = sh[k - 1];
  const bool a_inner_ok = as[k - 1] == 1 || as[k - 1] == 0;
  const bool b_inner_ok = bs_[k - 1] == 1 || bs_[k - 1] == 0;
  bool vec = (Q % 4 == 0) && a_inner_ok && b_inner_ok && n / 4 < 0xffffffffull && aligned16_h(y) &&
             !(as[k - 1] == 0 && bs_[k - 1] == 0);
  if (vec) {
    for (int d = 0; d < k - 1; ++d) {
      if (as[k - 1] == 1 && (as[d] % 4) != 0) vec = false;
      if (bs_[k - 1] == 1 && (bs_[d] % 4) != 0) vec = false;
    }
    if (as[k - 1] == 1 && !aligned16_h(a)) vec = false;
    if (bs_[k - 1] == 1 && !aligned16_h(b)) vec = false;
  }
  if (vec) {
    const uint32_t q4 = (uint32_t)(Q / 4);
    const uint32_t n4 = (uint32_t)(n / 4);
    const unsigned blocks = chunk_blocks(n4);
    // A full contiguous operand with a row-invariant other operand: row-vector kernel.
    bool a_rowinv = as[k - 1] == 1, b_rowinv = bs_[k - 1] == 1;
    for (int d = 0; d < k - 1; ++d) { if (as[d] != 0) a_rowinv = false; if (bs_[d] != 0) b_rowinv = false; }
    bool a_full = as[k - 1] == 1, b_full = bs_[k - 1] == 1;
    for (int d = 0; d + 1 < k; ++d) {
      if (as[d] != as[d + 1] * sh[d + 1]) a_full = false;
      if (bs_[d] != bs_[d + 1] * sh[d + 1]) b_full = false;
    }
    const FastDiv nc(q4);
    if (b_rowinv && a_full) {
      switch (op) {
#define X(OPC) case OPC: launch_pdl(k_rowvec_chunk<OPC, false, false>, dim3(blocks), dim3(256), 0, st, a, b, y, n4, nc); break;
        DCT_BCAST_CASES(X)
#undef X
        default: return cudaErrorInvalidValue;
      }
      return cudaGetLastError();
    }
    if (a_rowinv && b_full) {
      switch (op) {
#define X(OPC) case OPC: launch_pdl(k_rowvec_chunk<OPC, true, false>, dim3(blocks), dim3(256), 0, st, b, a, y, n4, nc); break;
        DCT_BCAST_CASES(X)
#undef X
        default: return cudaErrorInvalidValue;
      }
      return cudaGetLastError();
    }
    // [P, R, Q] with one operand constant along R and both contiguous along Q
    if (k == 3 && as[2] == 1 && bs_[2] == 1 && (as[1] == 0 || bs_[1] == 0) && sh[0] < 65536) {
      const bool swap = as[1] != 0;                 // B is the R-invariant operand
      const float* inv = swap ? b : a;
      const float* var = swap ? a : b;
      const int64_t sip = swap ? bs_[0] : as[0];
      const int64_t svp = swap ? as[0] : bs_[0];
      const int64_t svr = swap ? as[1] : bs_[1];
      const uint32_t R = (uint32_t)sh[1];
      const uint32_t gx = (q4 + 255) / 256;
      const DevInfo& di = dev_info();
      const uint64_t target = (uint64_t)di.sm_count * (di.max_threads_per_sm / 256) * 4;
      const uint64_t have = (uint64_t)gx * (uint64_t)sh[0];
      uint32_t chunks = (uint32_t)std::min<uint64_t>(R, std::max<uint64_t>(1, (target + have - 1) / have));
      if (chunks > 65535) chunks = 65535;
      const uint32_t rchunk = (R + chunks - 1) / chunks;
      const dim3 grid(gx, (R + rchunk - 1) / rchunk, (unsigned)sh[0]);
      switch (op) {
#define X(OPC)                                                                                         \
  case OPC:                                                                                            \
    if (swap) launch_pdl(k_bcast3<OPC, true>, dim3(grid), dim3(256), 0, st, inv, var, y, R, q4, rchunk, sip, svp, svr);     \
    else launch_pdl(k_bcast3<OPC, false>, dim3(grid), dim3(256), 0, st, inv, var, y, R, q4, rchunk, sip, svp, svr);        \
    break;
        DCT_BCAST_CASES(X)
#undef X
        default: return cudaErrorInvalidValue;
      }
      return cudaGetLastError();
    }
    RowMap m;
    m.nouter = k - 1;
    m.q4div = nc;
    for (int d = 0; d < k - 1; ++d) {
      const int src = k - 2 - d;                   // innermost outer dim first
      m.div[d] = FastDiv((uint32_t)sh[src]);
      m.a_str[d] = as[src];
      m.b_str[d] = bs_[src];
    }
    const bool abc = as[k - 1] == 0, bbc = bs_[k - 1] == 0;
    switch (op) {
#define X(OPC)                                                                                    \
  case OPC:                                                                                       \
    if (abc) launch_pdl(k_bcast_chunk<OPC, true, false>, dim3(blocks), dim3(256), 0, st, a, b, y, n4, m);              \
    else if (bbc) launch_pdl(k_bcast_chunk<OPC, false, true>, dim3(blocks), dim3(256), 0, st, a, b, y, n4, m);         \
    else launch_pdl(k_bcast_chunk<OPC, false, false>, dim3(blocks), dim3(256), 0, st, a, b, y, n4, m);                 \
    break;
      DCT_BCAST_CASES(X)
#undef X
      default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  if (n >= 0xffffffffull) return cudaErrorInvalidValue;
  ElemMap m;
  m.ndim = k;
  for (int d = 0; d < k; ++d) {
    const int src = k - 1 - d;
    m.div[d] = FastDiv((uint32_t)sh[src]);
    m.a_str[d] = as[src];
    m.b_str[d] = bs_[src];
  }
  const unsigned blocks = grid_for(n, 256);
  switch (op) {
#define X(OPC) case OPC: launch_pdl(k_bcast_scalar<OPC>, dim3(blocks), dim3(256), 0, st, a, b, y, n, m); break;
    DCT_BCAST_CASES(X)
#undef X
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// small reference-compat kernels
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_relu_bounded(const float* x, uint64_t n_in, float* y, uint64_t n_out) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_out; i += stride)
    y[i] = i < n_in ? unary_op<EW_RELU>(x[i], 0.f) : 0.0f;
}

cudaError_t launch_relu_bounded(const float* x, uint64_t n_in, float* y, uint64_t n_out, cudaStream_t st) {
  if (n_out == 0) return cudaSuccess;
  if (n_in >= n_out) return launch_unary(EW_RELU, x, y, n_out, 0.f, st);
  launch_pdl(k_relu_bounded, dim3(grid_for(n_out, 256)), dim3(256), 0, st, x, n_in, y, n_out);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_gap_bwd(const float* g, float* dx, uint64_t n, uint32_t S, FastDiv ds) {
  pdl_entry();
  const float fs = (float)S;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint64_t nc = i < 0xffffffffull ? ds.div((uint32_t)i) : i / S;
    dx[i] = __fdiv_rn(ld_keep(g + nc), fs);
  }
}

cudaError_t launch_gap_backward(const float* g, float* dx, uint64_t n, uint32_t S, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (S == 0) return cudaErrorInvalidValue;
  launch_pdl(k_gap_bwd, dim3(grid_for(n, 256)), dim3(256), 0, st, g, dx, n, S, FastDiv(S));
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_softmax_ce_grad(const float* p, const float* labels, float* grad,
                                                         uint32_t B, uint32_t K, uint32_t rows, uint32_t cols) {
  pdl_entry();
  const float fb = (float)B;
  for (uint32_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float lab = labels[r];
    const uint64_t base = (uint64_t)r * K;
    for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) {
      const float oh = (lab == (float)c) ? 1.0f : 0.0f;
      grad[base + c] = __fdiv_rn(__fsub_rn(p[base + c], oh), fb);
    }
  }
}

cudaError_t launch_softmax_ce_grad(const float* p, const float* labels, float* grad, uint32_t B, uint32_t K,
                                   uint32_t rows, uint32_t cols, cudaStream_t st) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  unsigned bs = cols >= 256 ? 256 : ((cols + 31) / 32) * 32;
  unsigned gx = (cols + bs - 1) / bs;
  unsigned gy = rows < 65535 ? rows : 65535;
  launch_pdl(k_softmax_ce_grad, dim3(dim3(gx, gy)), dim3(bs), 0, st, p, labels, grad, B, K, rows, cols);
  return cudaGetLastError();
}

__global__ void k_accumulate_scalar(const float* src, float* dst) {
  pdl_entry(); dst[0] = __fadd_rn(dst[0], src[0]); }

cudaError_t launch_accumulate_scalar(const float* src, float* dst, cudaStream_t st) {
  launch_pdl(k_accumulate_scalar, dim3(1), dim3(1), 0, st, src, dst);
  return cudaGetLastError();
}

// nn_dice_loss_grad.hlsl:17-34: dx[i] = -2 * (t[i] * denom - inter) / (denom * denom) / batch
// with (inter, sum p, sum t) of sample b = i / size and denom = sum p + sum t + 1e-6
// (the reference's gradient reads the target and the sums, not the prediction).
DCT_DEV float dice_grad1(float t, float inter, float denom, float fb) {
  const float num = __fmul_rn(-2.0f, __fsub_rn(__fmul_rn(t, denom), inter));
  return __fdiv_rn(__fdiv_rn(num, __fmul_rn(denom, denom)), fb);
}

DCT_DEV void dice_sample(const float* sums, uint64_t b, float& inter, float& denom) {
  inter = __ldg(sums + b * 3 + 0);
  denom = __fadd_rn(__fadd_rn(__ldg(sums + b * 3 + 1), __ldg(sums + b * 3 + 2)), 1e-6f);
}

// scalar form: any size, any alignment
__global__ void __launch_bounds__(256) k_dice_grad(const float* target, const float* sums, float* dx, uint32_t batch,
                                                   uint32_t size, uint64_t n) {
  pdl_entry();
  const float fb = (float)batch;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float inter, denom;
    dice_sample(sums, i / size, inter, denom);
    dx[i] = dice_grad1(target[i], inter, denom, fb);
  }
}

// the chunked float4 schedule (see the streaming kernels above) when size and n
// are multiples of 4 (a vector never straddles two samples) and the float4
// count fits 32 bits: the sample of float4 i is i / (size / 4), a fast division
__global__ void __launch_bounds__(256) k_dice_grad_chunk(const float* target, const float* sums, float* dx,
                                                         uint32_t batch, uint64_t n4, FastDiv per_sample4) {
  pdl_entry();
  const float fb = (float)batch;
  const uint64_t base = (uint64_t)blockIdx.x * kChunk4 + threadIdx.x;
  float4 v[kChunkU];
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) v[k] = ld_stream4(target + 4 * i);
  }
#pragma unroll
  for (int k = 0; k < kChunkU; ++k) {
    const uint64_t i = base + 256ull * k;
    if (i < n4) {
      float inter, denom;
      dice_sample(sums, per_sample4.div((uint32_t)i), inter, denom);
      st_stream4(dx + 4 * i, make_float4(dice_grad1(v[k].x, inter, denom, fb), dice_grad1(v[k].y, inter, denom, fb),
                                         dice_grad1(v[k].z, inter, denom, fb), dice_grad1(v[k].w, inter, denom, fb)));
    }
  }
}

cudaError_t launch_dice_grad(const float* pred, const float* target, const float* sums, float* dx,
                             uint32_t batch, uint32_t size, uint64_t n, cudaStream_t st) {
  (void)pred;
  if (n == 0) return cudaSuccess;
  if (size == 0 || batch == 0) return cudaErrorInvalidValue;
  const uint64_t n4 = n >> 2;
  if (size % 4 == 0 && n % 4 == 0 && n4 <= 0xffffffffull && aligned16_h(target) && aligned16_h(dx))
    launch_pdl(k_dice_grad_chunk, dim3(std::max(1u, chunk_blocks(n4))), dim3(256), 0, st, target, sums, dx, batch,
               n4, FastDiv(size / 4));
  else
    launch_pdl(k_dice_grad, dim3(grid_for(n, 256)), dim3(256), 0, st, target, sums, dx, batch, size, n);
  return cudaGetLastError();
}

}  // namespace dct
