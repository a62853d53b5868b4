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
// Design: grid-stride loops over 128-bit vectors with streaming cache hints,
// grids of (SMs x resident blocks); broadcast operands are resolved per ROW of
// the collapsed output (one division chain per row, amortised over the row),
// and a row-invariant operand vector is held in registers for all rows a
// thread visits.  All arithmetic uses the round-to-nearest intrinsics so no
// multiply-add is ever contracted: the results are bit-identical to the fp32
// formulas of the shaders / NumPy.
#include "dct_common.cuh"
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
    // 1/(1+exp(-x)); for x < 0 the equal form e/(1+e), e = exp(x), keeps the
    // relative error of exp instead of overflowing exp(-x) for x < -88.
    if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    float e = expf(x);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
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
// flat kernels (same shape).  Inputs may alias the output (in-place ops such as
// grad_accum / Muon's scale_add); every element is read and written by one
// thread, loads first.
// ---------------------------------------------------------------------------
constexpr int kUnroll = 4;

template <int OP>
__global__ void __launch_bounds__(256) k_unary_vec(const float* x, float* y, uint64_t n, float al) {
  const uint64_t n4 = n >> 2;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) v[k] = ld_stream4(x + 4 * (i + k * stride));
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) st_stream4(y + 4 * (i + k * stride), unary4<OP>(v[k], al));
  }
  for (; i < n4; i += stride) st_stream4(y + 4 * i, unary4<OP>(ld_stream4(x + 4 * i), al));
  const uint64_t t = 4 * n4 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) y[t] = unary_op<OP>(x[t], al);
}

template <int OP>
__global__ void __launch_bounds__(256) k_unary_scalar(const float* x, float* y, uint64_t n, float al) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = unary_op<OP>(x[i], al);
}

template <int OP>
__global__ void __launch_bounds__(256) k_binary_vec(const float* a, const float* b, float* y,
                                                    uint64_t n, float al, float be) {
  const uint64_t n4 = n >> 2;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      va[k] = ld_stream4(a + 4 * (i + k * stride));
      vb[k] = ld_stream4(b + 4 * (i + k * stride));
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) st_stream4(y + 4 * (i + k * stride), binary4<OP>(va[k], vb[k], al, be));
  }
  for (; i < n4; i += stride)
    st_stream4(y + 4 * i, binary4<OP>(ld_stream4(a + 4 * i), ld_stream4(b + 4 * i), al, be));
  const uint64_t t = 4 * n4 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) y[t] = binary_op<OP>(a[t], b[t], al, be);
}

template <int OP>
__global__ void __launch_bounds__(256) k_binary_scalar(const float* a, const float* b, float* y,
                                                       uint64_t n, float al, float be) {
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

// Vector path: Q % 4 == 0, all row bases 16-byte aligned for operands whose
// inner stride is 1.  A_BC / B_BC: operand broadcast along the inner dim.
// When the operand's row offset does not change between the rows a thread
// visits (stride-0 in every outer dim), its vector stays in registers.
template <int OP, bool A_BC, bool B_BC>
__global__ void __launch_bounds__(256) k_bcast_rows_vec(const float* __restrict__ a, const float* __restrict__ b,
                                                        float* __restrict__ y, uint32_t rows, uint32_t q4,
                                                        const __grid_constant__ RowMap m) {
  const uint32_t c4 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c4 >= q4) return;
  const uint64_t qn = 4ull * q4;
  for (uint32_t r = blockIdx.y; r < rows; r += gridDim.y) {
    int64_t ao, bo;
    row_offsets(m, r, ao, bo);
    float4 va, vb;
    if (A_BC) { float s = ld_keep(a + ao); va = make_float4(s, s, s, s); }
    else va = ld_keep4(a + ao + 4 * (int64_t)c4);
    if (B_BC) { float s = ld_keep(b + bo); vb = make_float4(s, s, s, s); }
    else vb = ld_keep4(b + bo + 4 * (int64_t)c4);
    st_stream4(y + (uint64_t)r * qn + 4ull * c4, binary4<OP>(va, vb, 0.f, 0.f));
  }
}

// Row broadcast with the broadcast row held in registers:
// y[r, c] = op(A[r, c], v[c]) (or op(v[c], A[r, c]) when SWAP), N % 4 == 0.
template <int OP, bool SWAP, bool RELU>
__global__ void __launch_bounds__(256) k_rowvec(const float* A, const float* v, float* y, uint32_t rows,
                                                uint32_t n4) {
  const uint32_t c4 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c4 >= n4) return;
  const float4 bv = ld_keep4(v + 4ull * c4);
  const uint64_t rn = 4ull * n4;
  uint32_t r = blockIdx.y;
  const uint32_t st = gridDim.y;
  for (; r + 3 * st < rows; r += 4 * st) {
    float4 x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = ld_stream4(A + (uint64_t)(r + k * st) * rn + 4ull * c4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float4 o = SWAP ? binary4<OP>(bv, x[k], 0.f, 0.f) : binary4<OP>(x[k], bv, 0.f, 0.f);
      if (RELU) o = unary4<EW_RELU>(o, 0.f);
      st_stream4(y + (uint64_t)(r + k * st) * rn + 4ull * c4, o);
    }
  }
  for (; r < rows; r += st) {
    float4 x = ld_stream4(A + (uint64_t)r * rn + 4ull * c4);
    float4 o = SWAP ? binary4<OP>(bv, x, 0.f, 0.f) : binary4<OP>(x, bv, 0.f, 0.f);
    if (RELU) o = unary4<EW_RELU>(o, 0.f);
    st_stream4(y + (uint64_t)r * rn + 4ull * c4, o);
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
  X(EW_RELU_GRAD) X(EW_RELU6_GRAD) X(EW_LEAKY_RELU_GRAD) X(EW_SIGMOID_GRAD) X(EW_SCALE_ADD)
#define DCT_BCAST_CASES(X) X(EW_ADD) X(EW_SUB) X(EW_MUL) X(EW_DIV) X(EW_MAXIMUM) X(EW_MINIMUM)

cudaError_t launch_unary(int op, const float* x, float* y, uint64_t n, float alpha, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const bool vec = aligned16_h(x) && aligned16_h(y);
  const unsigned blocks = grid_for(vec ? (n + 3) / 4 : n, 256);
  switch (op) {
#define X(OPC)                                                                      \
  case OPC:                                                                         \
    if (vec) k_unary_vec<OPC><<<blocks, 256, 0, st>>>(x, y, n, alpha);             \
    else k_unary_scalar<OPC><<<blocks, 256, 0, st>>>(x, y, n, alpha);              \
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
  const bool vec = aligned16_h(a) && aligned16_h(b) && aligned16_h(y);
  const unsigned blocks = grid_for(vec ? (n + 3) / 4 : n, 256);
  switch (op) {
#define X(OPC)                                                                        \
  case OPC:                                                                           \
    if (vec) k_binary_vec<OPC><<<blocks, 256, 0, st>>>(a, b, y, n, alpha, beta);     \
    else k_binary_scalar<OPC><<<blocks, 256, 0, st>>>(a, b, y, n, alpha, beta);      \
    break;
    DCT_BINARY_CASES(X)
#undef X
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

static void rowvec_geometry(uint32_t rows, uint32_t n4, dim3& grid, unsigned& bs) {
  bs = n4 >= 256 ? 256 : ((n4 + 31) / 32) * 32;
  if (bs == 0) bs = 32;
  const unsigned gx = (n4 + bs - 1) / bs;
  const DevInfo& d = dev_info();
  const uint64_t target = (uint64_t)d.sm_count * (d.max_threads_per_sm / bs);
  uint64_t gy = gx >= target ? 1 : target / gx;
  if (gy > rows) gy = rows;
  if (gy < 1) gy = 1;
  if (gy > 65535) gy = 65535;
  grid = dim3(gx, (unsigned)gy, 1);
}

cudaError_t launch_add_bias(const float* A, const float* B, float* C, uint64_t M, uint64_t N, bool relu,
                            cudaStream_t st) {
  const uint64_t n = M * N;
  if (n == 0) return cudaSuccess;
  if (N % 4 == 0 && M < 0xffffffffull && N / 4 < 0xffffffffull && aligned16_h(A) && aligned16_h(B) &&
      aligned16_h(C)) {
    dim3 grid; unsigned bs;
    rowvec_geometry((uint32_t)M, (uint32_t)(N / 4), grid, bs);
    if (relu) k_rowvec<EW_ADD, false, true><<<grid, bs, 0, st>>>(A, B, C, (uint32_t)M, (uint32_t)(N / 4));
    else k_rowvec<EW_ADD, false, false><<<grid, bs, 0, st>>>(A, B, C, (uint32_t)M, (uint32_t)(N / 4));
  } else {
    if (N == 0 || N > 0xffffffffull) return cudaErrorInvalidValue;
    const unsigned blocks = grid_for(n, 256);
    FastDiv dn((uint32_t)N);
    if (relu) k_add_bias_scalar<true><<<blocks, 256, 0, st>>>(A, B, C, n, (uint32_t)N, dn);
    else k_add_bias_scalar<false><<<blocks, 256, 0, st>>>(A, B, C, n, (uint32_t)N, dn);
  }
  return cudaGetLastError();
}

// Collapse adjacent output dims whose operand strides compose (both operands
// contiguous-with-broadcast), then pick the vector row kernel, the register-
// held row-vector kernel, or the scalar fallback.
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
  uint64_t rows = n / (uint64_t)Q;
  bool vec = (Q % 4 == 0) && a_inner_ok && b_inner_ok && rows < 0xffffffffull && aligned16_h(y) &&
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
    dim3 grid; unsigned bsz;
    rowvec_geometry((uint32_t)rows, q4, grid, bsz);
    // Row-invariant operand (stride 0 in all outer dims, contiguous inner): register-held kernel.
    bool a_rowinv = as[k - 1] == 1, b_rowinv = bs_[k - 1] == 1;
    for (int d = 0; d < k - 1; ++d) { if (as[d] != 0) a_rowinv = false; if (bs_[d] != 0) b_rowinv = false; }
    const bool a_full = as[k - 1] == 1 && (k == 1 || as[k - 2] == Q) ;
    const bool b_full = bs_[k - 1] == 1 && (k == 1 || bs_[k - 2] == Q);
    bool contiguous_rows_a = a_full, contiguous_rows_b = b_full;
    for (int d = 0; d + 1 < k - 1; ++d) {
      if (as[d] != as[d + 1] * sh[d + 1]) contiguous_rows_a = false;
      if (bs_[d] != bs_[d + 1] * sh[d + 1]) contiguous_rows_b = false;
    }
    if (b_rowinv && contiguous_rows_a) {
      switch (op) {
#define X(OPC) case OPC: k_rowvec<OPC, false, false><<<grid, bsz, 0, st>>>(a, b, y, (uint32_t)rows, q4); break;
        DCT_BCAST_CASES(X)
#undef X
        default: return cudaErrorInvalidValue;
      }
      return cudaGetLastError();
    }
    if (a_rowinv && contiguous_rows_b) {
      switch (op) {
#define X(OPC) case OPC: k_rowvec<OPC, true, false><<<grid, bsz, 0, st>>>(b, a, y, (uint32_t)rows, q4); break;
        DCT_BCAST_CASES(X)
#undef X
        default: return cudaErrorInvalidValue;
      }
      return cudaGetLastError();
    }
    RowMap m;
    m.nouter = k - 1;
    for (int d = 0; d < k - 1; ++d) {
      const int src = k - 2 - d;                   // innermost outer dim first
      m.div[d] = FastDiv((uint32_t)sh[src]);
      m.a_str[d] = as[src];
      m.b_str[d] = bs_[src];
    }
    const bool abc = as[k - 1] == 0, bbc = bs_[k - 1] == 0;
    switch (op) {
#define X(OPC)                                                                                         \
  case OPC:                                                                                            \
    if (abc) k_bcast_rows_vec<OPC, true, false><<<grid, bsz, 0, st>>>(a, b, y, (uint32_t)rows, q4, m);  \
    else if (bbc) k_bcast_rows_vec<OPC, false, true><<<grid, bsz, 0, st>>>(a, b, y, (uint32_t)rows, q4, m); \
    else k_bcast_rows_vec<OPC, false, false><<<grid, bsz, 0, st>>>(a, b, y, (uint32_t)rows, q4, m);    \
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
#define X(OPC) case OPC: k_bcast_scalar<OPC><<<blocks, 256, 0, st>>>(a, b, y, n, m); break;
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
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_out; i += stride)
    y[i] = i < n_in ? unary_op<EW_RELU>(x[i], 0.f) : 0.0f;
}

cudaError_t launch_relu_bounded(const float* x, uint64_t n_in, float* y, uint64_t n_out, cudaStream_t st) {
  if (n_out == 0) return cudaSuccess;
  if (n_in >= n_out) return launch_unary(EW_RELU, x, y, n_out, 0.f, st);
  k_relu_bounded<<<grid_for(n_out, 256), 256, 0, st>>>(x, n_in, y, n_out);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_gap_bwd(const float* g, float* dx, uint64_t n, uint32_t S, FastDiv ds) {
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
  k_gap_bwd<<<grid_for(n, 256), 256, 0, st>>>(g, dx, n, S, FastDiv(S));
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_softmax_ce_grad(const float* p, const float* labels, float* grad,
                                                         uint32_t B, uint32_t K, uint32_t rows, uint32_t cols) {
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
  k_softmax_ce_grad<<<dim3(gx, gy), bs, 0, st>>>(p, labels, grad, B, K, rows, cols);
  return cudaGetLastError();
}

__global__ void k_accumulate_scalar(const float* src, float* dst) { dst[0] = __fadd_rn(dst[0], src[0]); }

cudaError_t launch_accumulate_scalar(const float* src, float* dst, cudaStream_t st) {
  k_accumulate_scalar<<<1, 1, 0, st>>>(src, dst);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_dice_grad(const float* pred, const float* target, const float* sums,
                                                   float* dx, uint32_t batch, uint32_t size, uint64_t n) {
  const float fb = (float)batch;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint64_t b = i / size;
    const float inter = sums[b * 3 + 0];
    const float denom = __fadd_rn(__fadd_rn(sums[b * 3 + 1], sums[b * 3 + 2]), 1e-6f);
    const float t = target[i];
    const float num = __fmul_rn(-2.0f, __fsub_rn(__fmul_rn(t, denom), inter));
    dx[i] = __fdiv_rn(__fdiv_rn(num, __fmul_rn(denom, denom)), fb);
  }
  (void)pred;
}

cudaError_t launch_dice_grad(const float* pred, const float* target, const float* sums, float* dx,
                             uint32_t batch, uint32_t size, uint64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (size == 0 || batch == 0) return cudaErrorInvalidValue;
  k_dice_grad<<<grid_for(n, 256), 256, 0, st>>>(pred, target, sums, dx, batch, size, n);
  return cudaGetLastError();
}

}  // namespace dct
