// Reduction kernels of libdct_cuda (sm_100a).
//
// Replaces the reference's one-group-per-output reductions (nn_bias_grad.hlsl:8-29,
// nn_global_avg_pool.hlsl:16-35, nn_rms.hlsl:7-24, nn_grad_sq_reduce.hlsl:16-30,
// nn_grad_norm_final.hlsl:16-35, nn_dice_loss_sums.hlsl:19-55) and adds NumPy
// axis / full reductions (sum, mean, max, argmax, min, argmin).
//
// Every sum accumulates in float64 (fp32 inputs convert exactly) and is rounded
// once at the store: the 0.1% +-1e4 outliers of the reduction benchmark would
// otherwise cancel digits of an fp32 accumulator.  Every combine runs in a
// fixed order (warp shuffle tree, then warps in index order, then chunk
// partials in index order), so results are bit-reproducible run to run on a
// given GPU.
//
// Shapes are handled as a strided 3-D view x[o*so + l*sl + i*si] reduced over l:
//  * si unused (inner == 1) and sl == 1: ROW kernel -- a warp streams one
//    (row, chunk) with 128-bit loads; long rows split into chunks whose
//    partials a second launch folds in order;
//  * si == 1: COLUMN kernel -- a block owns 32 (x4) adjacent columns, its 8
//    warps walk interleaved rows (each warp load is 512 contiguous bytes), the
//    8 per-warp accumulators combine through shared memory; the reduced axis is
//    split into chunks when there are too few column tiles to fill the GPU;
//  * anything else: one thread per output.
#include <algorithm>

#include "dct_common.cuh"
#include "dct_fold.cuh"
#include "kernels.h"

namespace dct {

namespace {

constexpr int kRedThreads = 256;
constexpr int kSumMaxDims = 8;
constexpr int kRedWarps = kRedThreads / 32;

// max / min that return NaN if either operand is NaN (one instruction)
DCT_DEV float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
DCT_DEV float fmin_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Where a finished reduction goes: float values (+ int32 indices), or, for a
// shard of a reduction split across ranks, one packed 8-byte partial per output
// with the shard's global index offset applied to arg indices.
struct RedOut {
  float* out = nullptr;
  int32_t* idx = nullptr;
  unsigned long long* packed = nullptr;
  int32_t idx_off = 0;
  // sums only: also acc[k] = acc[k] + out[k] in float32 (nn_grad_accum.hlsl:5-8
  // on the stored value, as a grad_accum dispatch after the reduction would)
  float* acc = nullptr;
};

// Partial accumulator of one reduction lane.
//  * sums: float64;
//  * MAX / MIN: value only, NaN propagates (NumPy);
//  * ARGMAX / ARGMIN: (value, int32 index); within one lane indices only grow,
//    so a later candidate replaces the current one only if strictly better
//    (a first NaN beats every number); merges of lanes, warps and chunks use
//    the full rule, ties going to the lower index.
template <int OP>
struct Acc {
  static constexpr bool kArg = (OP == RED_ARGMAX || OP == RED_ARGMIN);
  static constexpr bool kExt = (OP == RED_MAX || OP == RED_MIN);
  static constexpr bool kMax = (OP == RED_MAX || OP == RED_ARGMAX);
  double s = 0.0;
  float v = kMax ? -INFINITY : INFINITY;
  int32_t i = -1;
  // the identity element (also the state of a lane that saw no input)
  DCT_DEV void reset() {
    s = 0.0;
    v = kMax ? -INFINITY : INFINITY;
    i = -1;
  }
  DCT_DEV static unsigned long long identity_pack() {
    Acc a;
    a.reset();
    return a.pack();
  }
  DCT_DEV void add(float x, int64_t idx) {
    if constexpr (kArg) {
      // common path: one compare (x <= v is false for a better x and for any NaN)
      if (i < 0 || !(kMax ? (x <= v) : (x >= v))) {
        const bool take = (i < 0) | (kMax ? (x > v) : (x < v)) | ((x != x) & (v == v));
        if (take) { v = x; i = (int32_t)idx; }
      }
    } else if constexpr (kExt) {
      v = kMax ? fmax_nan(v, x) : fmin_nan(v, x);
    } else if constexpr (OP == RED_SUMSQ) {
      double d = (double)x;
      s += d * d;
    } else {
      s += (double)x;
    }
  }
  DCT_DEV void merge(const Acc& o) {
    if constexpr (kArg) {
      if (o.i >= 0 && (i < 0 || better<kMax>(o.v, o.i, v, i))) { v = o.v; i = o.i; }
    } else if constexpr (kExt) {
      v = ((kMax ? (o.v > v) : (o.v < v)) || (o.v != o.v)) && !(v != v) ? o.v : v;
    } else {
      s += o.s;
    }
  }
  DCT_DEV void warp_reduce() {
    if constexpr (kArg) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        Acc o;
        o.v = __shfl_down_sync(0xffffffffu, v, off);
        o.i = __shfl_down_sync(0xffffffffu, i, off);
        merge(o);
      }
    } else if constexpr (kExt) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        Acc o;
        o.v = __shfl_down_sync(0xffffffffu, v, off);
        merge(o);
      }
    } else {
      s = warp_sum(s);
    }
  }
  // packed 8-byte partial
  DCT_DEV unsigned long long pack() const {
    if constexpr (kArg || kExt) {
      return ((unsigned long long)(uint32_t)__float_as_uint(v) << 32) | (uint32_t)i;
    } else {
      return (unsigned long long)__double_as_longlong(s);
    }
  }
  DCT_DEV void unpack(unsigned long long w) {
    if constexpr (kArg || kExt) {
      v = __uint_as_float((uint32_t)(w >> 32));
      i = (int32_t)(uint32_t)(w & 0xffffffffu);
    } else {
      s = __longlong_as_double((long long)w);
    }
  }
  DCT_DEV void emit(const RedOut& o, uint64_t k, uint64_t len) const {
    if (o.packed) {
      Acc t = *this;
      if constexpr (kArg) { if (t.i >= 0) t.i += o.idx_off; }
      o.packed[k] = t.pack();
    } else {
      store(o.out, o.idx, k, len);
      if constexpr (!kArg && !kExt) {
        if (o.acc) o.acc[k] = __fadd_rn(o.acc[k], o.out[k]);
      }
    }
  }
  DCT_DEV void store(float* out, int32_t* out_idx, uint64_t k, uint64_t len) const {
    if constexpr (kArg) {
      if (out) out[k] = v;
      if (out_idx) out_idx[k] = i;
    } else if constexpr (kExt) {
      out[k] = v;
    } else if constexpr (OP == RED_MEAN) {
      out[k] = (float)(s / (double)len);
    } else {
      out[k] = (float)s;
    }
  }
};

// Streaming state of one column in the column kernel's hot loop, cheaper per
// element than Acc: sums add in float64; max / min use the NaN-propagating
// instruction; arg reductions keep (value, row) updated only on a strictly
// better value -- rows arrive in increasing order, so that is the first
// occurrence -- and a NaN flag.  A lane that saw a NaN rescans its own rows for
// the first NaN afterwards (NaN is the maximum and the minimum).  The lane
// starts at its first row, so an all -inf (+inf) column still names that row.
template <int OP>
struct ColLane {
  static constexpr bool kArg = Acc<OP>::kArg;
  static constexpr bool kExt = Acc<OP>::kExt;
  static constexpr bool kMax = Acc<OP>::kMax;
  double s;
  float v;
  int32_t i;
  DCT_DEV void reset(int32_t first_row) {
    s = 0.0;
    v = kMax ? -INFINITY : INFINITY;
    i = first_row;
  }
  DCT_DEV void add(float x, int32_t row) {
    if constexpr (kArg) {
      // three instructions: the NaN-propagating extreme is both the running
      // value (equal to the strict-better one while no NaN was seen) and the
      // NaN flag (once NaN, no later element is better and finish() rescans)
      const bool u = kMax ? (x > v) : (x < v);
      i = u ? row : i;
      v = kMax ? fmax_nan(v, x) : fmin_nan(v, x);
    } else if constexpr (kExt) {
      v = kMax ? fmax_nan(v, x) : fmin_nan(v, x);
    } else if constexpr (OP == RED_SUMSQ) {
      const double d = (double)x;
      s = fma(d, d, s);
    } else {
      s += (double)x;
    }
  }
  // Acc form of this lane; `col` is the lane's column pointer (row 0), rows
  // first_row, first_row + step, ... < end were visited (`seen` false: none).
  DCT_DEV Acc<OP> finish(const float* col, uint64_t sl, uint64_t first_row, uint64_t step, uint64_t end,
                         bool seen) const {
    Acc<OP> a;
    a.reset();
    if (!seen) return a;
    if constexpr (kArg) {
      a.v = v;
      a.i = i;
      if (v != v) {                                       // rare: find this lane's first NaN
        for (uint64_t r = first_row; r < end; r += step) {
          const float x = col[r * sl];
          if (x != x) { a.v = x; a.i = (int32_t)r; break; }
        }
      }
    } else if constexpr (kExt) {
      a.v = v;
    } else {
      a.s = s;
    }
    return a;
  }
  // Acc form for the row kernel's lanes: indices first + 128 t + q (q < 4), < end
  DCT_DEV Acc<OP> finish_rows(const float* row, uint64_t first, uint64_t end, uint64_t step = 128) const {
    Acc<OP> a;
    a.reset();
    if (first >= end) return a;
    if constexpr (kArg) {
      a.v = v;
      a.i = i;
      if (v != v) {                                       // rare: this lane's first NaN
        for (uint64_t l = first; l < end; l += step) {
          bool found = false;
          for (int q = 0; q < 4 && l + q < end; ++q) {
            const float xq = row[l + q];
            if (xq != xq) { a.v = xq; a.i = (int32_t)(l + q); found = true; break; }
          }
          if (found) break;
        }
      }
    } else if constexpr (kExt) {
      a.v = v;
    } else {
      a.s = s;
    }
    return a;
  }
};

// ---------------------------------------------------------------------------
// ROW kernel: (row, chunk) per warp, contiguous along the reduced axis.
// ---------------------------------------------------------------------------
template <int OP, bool VEC>
__global__ void __launch_bounds__(kRedThreads) k_reduce_rows(const float* __restrict__ x, uint64_t rows, uint64_t len,
                                                             uint64_t so, uint32_t chunks, uint64_t chunk_len,
                                                             RedOut ro, unsigned long long* part) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint64_t pairs = rows * chunks;
  for (uint64_t pr = gw; pr < pairs; pr += nw) {
    const uint64_t row = pr / chunks;
    const uint32_t ch = (uint32_t)(pr - row * chunks);
    const uint64_t l0 = (uint64_t)ch * chunk_len;
    const uint64_t l1 = min(len, l0 + chunk_len);
    const float* p = x + row * so;
    Acc<OP> acc;
    acc.reset();
    if (VEC) {
      // lane-local streaming state (see ColLane): the lane visits its indices in
      // increasing order, 4 consecutive per float4
      const uint64_t first = l0 + 4 * (uint64_t)lane;
      ColLane<OP> ln;
      ln.reset((int32_t)first);
      uint64_t l = first;
      for (; l + 3 * 128 + 3 < l1; l += 4 * 128) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = ld_stream4(p + l + 128 * k);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int32_t b = (int32_t)(l + 128 * k);
          ln.add(v[k].x, b); ln.add(v[k].y, b + 1); ln.add(v[k].z, b + 2); ln.add(v[k].w, b + 3);
        }
      }
      for (; l + 3 < l1; l += 128) {
        const float4 v = ld_stream4(p + l);
        const int32_t b = (int32_t)l;
        ln.add(v.x, b); ln.add(v.y, b + 1); ln.add(v.z, b + 2); ln.add(v.w, b + 3);
      }
      acc = ln.finish_rows(p, first, l1);
    } else {
      for (uint64_t l = l0 + lane; l < l1; l += 32) acc.add(ld_stream(p + l), (int64_t)l);
    }
    acc.warp_reduce();
    if (lane == 0) {
      if (chunks == 1) acc.emit(ro, row, len);
      else part[pr] = acc.pack();
    }
  }
}

// ---------------------------------------------------------------------------
// ROW kernel, one block per row: for rows that fill a quarter of the warp
// slots or less (a one-warp-per-row grid would leave most SMs idle).  The
// block's 256 threads stream the row -- thread t the float4s 4t, 4t + 1024, ...
// in increasing order, so the lane-local state of the row kernel applies --
// then each warp reduces its lanes and warp 0 merges the 8 warp results in
// warp order: one launch, no chunk partials, no fold.
// ---------------------------------------------------------------------------
template <int OP, bool VEC>
__global__ void __launch_bounds__(kRedThreads) k_reduce_rows_block(const float* __restrict__ x, uint64_t rows,
                                                                   uint64_t len, uint64_t so, RedOut ro) {
  pdl_entry();
  __shared__ unsigned long long sh[kRedWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr uint64_t T = kRedThreads;
  for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* p = x + row * so;
    Acc<OP> acc;
    acc.reset();
    if (VEC) {
      const uint64_t first = 4 * (uint64_t)threadIdx.x;
      ColLane<OP> ln;
      ln.reset((int32_t)first);
      uint64_t l = first;
      for (; l + 3 * 4 * T + 3 < len; l += 4 * 4 * T) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = ld_stream4(p + l + 4 * T * k);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int32_t b = (int32_t)(l + 4 * T * k);
          ln.add(v[k].x, b); ln.add(v[k].y, b + 1); ln.add(v[k].z, b + 2); ln.add(v[k].w, b + 3);
        }
      }
      for (; l + 3 < len; l += 4 * T) {
        const float4 v = ld_stream4(p + l);
        const int32_t b = (int32_t)l;
        ln.add(v.x, b); ln.add(v.y, b + 1); ln.add(v.z, b + 2); ln.add(v.w, b + 3);
      }
      acc = ln.finish_rows(p, first, len, 4 * T);
    } else {
      for (uint64_t l = threadIdx.x; l < len; l += T) acc.add(ld_stream(p + l), (int64_t)l);
    }
    acc.warp_reduce();
    if (lane == 0) sh[warp] = acc.pack();
    __syncthreads();
    if (warp == 0) {
      Acc<OP> tot;
      const unsigned long long mine = lane < kRedWarps ? sh[lane] : 0ull;
#pragma unroll
      for (int w = 0; w < kRedWarps; ++w) {
        Acc<OP> t;
        t.unpack(__shfl_sync(0xffffffffu, mine, w));
        if (w == 0) tot = t; else tot.merge(t);
      }
      if (lane == 0) tot.emit(ro, row, len);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// COLUMN kernel: block = 32*VEC adjacent outputs x 8 interleaved row lanes.
// grid = (column tiles, outer (strided), len chunks)
// ---------------------------------------------------------------------------
// With chunks > 1 each block leaves its tile's partial for its chunk; a fold
// kernel launched with programmatic dependent launch combines them in chunk
// order.  (A fold by the last block of each tile, found with an atomic counter,
// was measured slower: its fence and serial fold sit on the kernel's tail.)
//
// MODE fuses an elementwise pass over the reduced matrix into the column sum,
// storing the transformed value to `out` (x's layout) as it streams by:
//  * COL_RELU_GRAD, the backward of bias + ReLU (nn_engine.py:1091-1106):
//    v = aux > 0 ? x : 0 with aux the forward output (relu_grad,
//    nn_relu_grad.hlsl:6-9), out = dx; the column sums are bias_grad
//    (nn_bias_grad.hlsl:8-29) of dx;
//  * COL_BIAS_RELU, the forward: v = max(0, x + aux[c]) with aux the bias row
//    (bias_relu, nn_bias_relu.hlsl:8-12), out = y; the column sums are
//    bias_grad of y.
// One read of the operands instead of two passes.  The per-lane order of the
// adds is the plain kernel's, so for the same plan the sums are bit-identical
// to the elementwise dispatch followed by bias_grad.
enum ColMode : int { COL_PLAIN = 0, COL_RELU_GRAD = 1, COL_BIAS_RELU = 2 };
struct ColXform {
  const float* aux = nullptr;   // COL_RELU_GRAD: the forward output; COL_BIAS_RELU: the bias row
  float* out = nullptr;         // the transformed matrix
};

DCT_DEV float relu_gate(float g, float y) { return y > 0.0f ? g : 0.0f; }
DCT_DEV float bias_relu1(float x, float b) {
  const float o = __fadd_rn(x, b);
  return o > 0.0f ? o : 0.0f;                           // HLSL max(0, x): NaN -> 0
}

template <int OP, int VEC, int MODE = COL_PLAIN>
__global__ void __launch_bounds__(kRedThreads) k_reduce_cols(const float* __restrict__ x, uint64_t outer, uint64_t len,
                                                             uint64_t inner, uint64_t so, uint64_t sl,
                                                             uint32_t chunks, uint64_t chunk_len, RedOut ro,
                                                             unsigned long long* part, ColXform xf) {
  pdl_entry();
  constexpr int W = 32 * VEC;
  constexpr bool GATE = MODE == COL_RELU_GRAD, BIAS = MODE == COL_BIAS_RELU, XF = MODE != COL_PLAIN;
  __shared__ unsigned long long sh[kRedWarps][W];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t c0 = (uint64_t)blockIdx.x * W + (uint64_t)lane * VEC;
  const uint32_t ch = blockIdx.z;
  const uint64_t l0 = (uint64_t)ch * chunk_len;
  const uint64_t l1 = min(len, l0 + chunk_len);
  for (uint64_t o = blockIdx.y; o < outer; o += gridDim.y) {
    Acc<OP> acc[VEC];
    const float* base = x + o * so;
    const float* ybase = GATE ? xf.aux + o * so : nullptr;
    float* dbase = XF ? xf.out + o * so : nullptr;
    if (VEC == 4 && c0 + 3 < inner) {
      // 8 rows (8 x 512 B per warp) in flight per batch: the loop is bound by
      // memory latency, not by the per-element work.  With a fused elementwise
      // pass, which also stores (and gated, loads a second operand), 4 rows.
      constexpr int U = XF ? 4 : 8;
      const float4 bv = BIAS ? ld_keep4(xf.aux + c0) : make_float4(0.f, 0.f, 0.f, 0.f);
      const uint64_t first = l0 + warp;
      ColLane<OP> ln[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) ln[j].reset((int32_t)first);
      uint64_t l = first;
      for (; l + (U - 1) * kRedWarps < l1; l += U * kRedWarps) {
        float4 v[U];
#pragma unroll
        for (int k = 0; k < U; ++k) v[k] = ld_stream4(base + (l + k * kRedWarps) * sl + c0);
        if constexpr (GATE) {
          float4 yv[U];
#pragma unroll
          for (int k = 0; k < U; ++k) yv[k] = ld_stream4(ybase + (l + k * kRedWarps) * sl + c0);
#pragma unroll
          for (int k = 0; k < U; ++k)
            v[k] = make_float4(relu_gate(v[k].x, yv[k].x), relu_gate(v[k].y, yv[k].y), relu_gate(v[k].z, yv[k].z),
                               relu_gate(v[k].w, yv[k].w));
        }
        if constexpr (BIAS) {
#pragma unroll
          for (int k = 0; k < U; ++k)
            v[k] = make_float4(bias_relu1(v[k].x, bv.x), bias_relu1(v[k].y, bv.y), bias_relu1(v[k].z, bv.z),
                               bias_relu1(v[k].w, bv.w));
        }
        if constexpr (XF) {
#pragma unroll
          for (int k = 0; k < U; ++k) st_stream4(dbase + (l + k * kRedWarps) * sl + c0, v[k]);
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int32_t li = (int32_t)(l + k * kRedWarps);
          ln[0].add(v[k].x, li); ln[1].add(v[k].y, li); ln[2].add(v[k].z, li); ln[3].add(v[k].w, li);
        }
      }
      for (; l < l1; l += kRedWarps) {
        float4 v = ld_stream4(base + l * sl + c0);
        if constexpr (GATE) {
          const float4 yv = ld_stream4(ybase + l * sl + c0);
          v = make_float4(relu_gate(v.x, yv.x), relu_gate(v.y, yv.y), relu_gate(v.z, yv.z), relu_gate(v.w, yv.w));
        }
        if constexpr (BIAS)
          v = make_float4(bias_relu1(v.x, bv.x), bias_relu1(v.y, bv.y), bias_relu1(v.z, bv.z), bias_relu1(v.w, bv.w));
        if constexpr (XF) st_stream4(dbase + l * sl + c0, v);
        const int32_t li = (int32_t)l;
        ln[0].add(v.x, li); ln[1].add(v.y, li); ln[2].add(v.z, li); ln[3].add(v.w, li);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[j < VEC ? j : 0] = ln[j].finish(base + c0 + j, sl, first, kRedWarps, l1, first < l1);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        if (c0 + j >= inner) break;
        const float bj = BIAS ? ld_keep(xf.aux + c0 + j) : 0.0f;
        for (uint64_t l = l0 + warp; l < l1; l += kRedWarps) {
          float v = ld_stream(base + l * sl + c0 + j);
          if constexpr (GATE) v = relu_gate(v, ld_stream(ybase + l * sl + c0 + j));
          if constexpr (BIAS) v = bias_relu1(v, bj);
          if constexpr (XF) st_stream(dbase + l * sl + c0 + j, v);
          acc[j].add(v, (int64_t)l);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) sh[warp][lane * VEC + j] = acc[j].pack();
    __syncthreads();
    if (threadIdx.x < W) {
      const uint64_t c = (uint64_t)blockIdx.x * W + threadIdx.x;
      Acc<OP> tot;
      for (int w = 0; w < kRedWarps; ++w) {
        Acc<OP> t;
        t.unpack(sh[w][threadIdx.x]);
        if (w == 0) tot = t; else tot.merge(t);
      }
      if (c < inner) {
        if (chunks == 1) tot.emit(ro, o * inner + c, len);
        else part[(o * chunks + ch) * inner + c] = tot.pack();
      }
    }
    __syncthreads();
  }
}

// Fold chunk partials: out[k] = combine over ch of part[(o*chunks + ch)*inner + c]
// (k = o*inner + c).  A block takes 32 adjacent outputs, one per lane; warp w
// folds chunks w, w+8, ... of its lane's output in order (each warp load reads
// one chunk's 32 adjacent partials: 256 contiguous bytes), then warp 0 merges
// the 8 warp partials in warp order, so the result is the same on every run
// (sums in float64; arg and extreme merges are exact).  The earlier form, a
// warp per output with lane l folding chunks l, l+32, ..., read one 8-byte
// word per 32-byte sector.
template <int OP>
__global__ void __launch_bounds__(256) k_fold_chunks(const unsigned long long* __restrict__ part, uint64_t nout,
                                                     uint32_t chunks, uint64_t inner, uint64_t len, RedOut ro) {
  pdl_entry();
  __shared__ unsigned long long sh[kRedWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint64_t k0 = (uint64_t)blockIdx.x * 32; k0 < nout; k0 += (uint64_t)gridDim.x * 32) {
    const uint64_t k = k0 + lane;
    Acc<OP> a;
    a.reset();
    if (k < nout) {
      const uint64_t o = k / inner, c = k - o * inner;
      const unsigned long long* p = part + o * chunks * inner + c;
#pragma unroll 4
      for (uint32_t ch = warp; ch < chunks; ch += kRedWarps) {
        Acc<OP> t;
        t.unpack(__ldcg(p + (uint64_t)ch * inner));
        a.merge(t);
      }
    }
    sh[warp][lane] = a.pack();
    __syncthreads();
    if (warp == 0 && k < nout) {
      Acc<OP> tot;
      tot.unpack(sh[0][lane]);
#pragma unroll
      for (int w = 1; w < kRedWarps; ++w) {
        Acc<OP> t;
        t.unpack(sh[w][lane]);
        tot.merge(t);
      }
      tot.emit(ro, k, len);
    }
    __syncthreads();
  }
}

// The last stage of a sharded axis reduction whose plan has more than one
// chunk, in the same launch as the exchange over peer memory (dct_peer.cuh):
// lane l of warp 0 folds column k's chunk partials as k_fold_chunks does,
// stores this rank's packed partial (global index) into every peer's slot,
// then merges every rank's partial for k in rank order as each arrives (ties
// to the lower index; mean divides by len_total) and emits.  The grid's last
// block does no tile: it stores the header, waits for every peer's (the slot
// reuse ordering) and checks that the shards tile the axis, off the tile
// blocks' path (as block 0's tail it cost 1.2 us per call).  The launch keeps
// the tile blocks resident, since each waits for the peers' puts.
template <int OP>
__global__ void __launch_bounds__(256) k_fold_chunks_xchg(const unsigned long long* __restrict__ part, uint64_t nout,
                                                          uint32_t chunks, uint64_t inner, uint64_t len_total,
                                                          int32_t idx_off, RedOut fin,
                                                          const __grid_constant__ PeerXfer p) {
  pdl_entry();
  bool gave_up = false;
  const unsigned tiles_grid = gridDim.x - 1;
  if (blockIdx.x == tiles_grid) {
    peer_put_header(p, true);
    peer_sync(p, gave_up, true);
    peer_check_axis(p, gave_up, true);
    return;
  }
  __shared__ unsigned long long sh[kRedWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint64_t k0 = (uint64_t)blockIdx.x * 32; k0 < nout; k0 += (uint64_t)tiles_grid * 32) {
    const uint64_t k = k0 + lane;
    Acc<OP> a;
    a.reset();
    if (k < nout) {
      const uint64_t o = k / inner, c = k - o * inner;
      const unsigned long long* q = part + o * chunks * inner + c;
#pragma unroll 4
      for (uint32_t ch = warp; ch < chunks; ch += kRedWarps) {
        Acc<OP> t;
        t.unpack(__ldcg(q + (uint64_t)ch * inner));
        a.merge(t);
      }
    }
    sh[warp][lane] = a.pack();
    __syncthreads();
    if (warp == 0 && k < nout) {
      Acc<OP> tot;
      tot.unpack(sh[0][lane]);
#pragma unroll
      for (int w = 1; w < kRedWarps; ++w) {
        Acc<OP> t;
        t.unpack(sh[w][lane]);
        tot.merge(t);
      }
      if constexpr (Acc<OP>::kArg) { if (tot.i >= 0) tot.i += idx_off; }
      const unsigned long long mine = tot.pack();
      peer_put_word(p, k, mine);
      Acc<OP> g;
      g.reset();
      for (int r = 0; r < p.world; ++r) {
        Acc<OP> t;
        t.unpack(r == p.rank ? mine : peer_get(p, r, k, gave_up));
        g.merge(t);
      }
      if (fin.out || fin.idx) g.emit(fin, k, len_total);
    }
    __syncthreads();
  }
}

// generic strided: one thread per output
template <int OP>
__global__ void __launch_bounds__(256) k_reduce_generic(const float* __restrict__ x, uint64_t outer, uint64_t len,
                                                        uint64_t inner, uint64_t so, uint64_t sl, uint64_t si,
                                                        RedOut ro) {
  pdl_entry();
  const uint64_t nout = outer * inner;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nout; k += stride) {
    const uint64_t o = k / inner, c = k - o * inner;
    const float* p = x + o * so + c * si;
    Acc<OP> acc;
    acc.reset();
    for (uint64_t l = 0; l < len; ++l) acc.add(p[l * sl], (int64_t)l);
    acc.emit(ro, k, len);
  }
}

struct Plan {
  int kind;           // 0 rows (a warp per row chunk), 1 cols, 2 generic, 3 rows (a block per row)
  bool vec;
  uint32_t chunks;
  uint64_t chunk_len;
  dim3 grid;
};

// cols_per_sm: resident blocks per SM of the column kernel that will run (its
// occupancy); the column plan fills exactly that many blocks per SM in one wave.
// Workspace sizing passes the largest possible value (every block resident).
Plan make_plan(uint64_t outer, uint64_t len, uint64_t inner, uint64_t so, uint64_t sl, uint64_t si,
               const float* x, int cols_per_sm = 0) {
  Plan p{};
  const DevInfo& d = dev_info();
  const uint64_t target_blocks = (uint64_t)d.sm_count * (d.max_threads_per_sm / kRedThreads);
  const uint64_t col_blocks =
      (uint64_t)d.sm_count * (cols_per_sm > 0 ? (uint64_t)cols_per_sm : (uint64_t)(d.max_threads_per_sm / kRedThreads));
  if (inner == 1 && sl == 1) {
    p.kind = 0;
    p.vec = (len % 4 == 0) && (so % 4 == 0) && aligned16_h(x);
    const uint64_t target_warps = target_blocks * kRedWarps * 2;
    uint64_t chunks = 1;
    if (outer < target_warps && len > 8192) {
      chunks = (target_warps + outer - 1) / outer;
      const uint64_t max_chunks = (len + 4095) / 4096;       // keep >= 4096 elements per chunk
      if (chunks > max_chunks) chunks = max_chunks;
    } else if (outer * 4 < target_warps && len >= 2048) {
      // few rows (a quarter of the warp slots or less): a block of 8 warps per
      // row (k_reduce_rows_block), one launch and no fold
      p.kind = 3;
      p.chunks = 1;
      p.chunk_len = len;
      p.grid = dim3((unsigned)(outer < target_blocks * 4 ? outer : target_blocks * 4), 1, 1);
      return p;
    }
    uint64_t cl = (len + chunks - 1) / chunks;
    cl = (cl + 3) & ~3ull;
    if (cl == 0) cl = 4;                                      // len 0: one empty chunk
    chunks = len ? (len + cl - 1) / cl : 1;
    p.chunks = (uint32_t)chunks;
    p.chunk_len = cl;
    const uint64_t warps = outer * chunks;
    uint64_t blocks = (warps + kRedWarps - 1) / kRedWarps;
    if (blocks > target_blocks * 4) blocks = target_blocks * 4;
    p.grid = dim3((unsigned)blocks, 1, 1);
  } else if (si == 1) {
    p.kind = 1;
    p.vec = (inner % 4 == 0) && (sl % 4 == 0) && (so % 4 == 0) && aligned16_h(x);
    const uint64_t W = p.vec ? 128 : 32;
    const uint64_t tiles = (inner + W - 1) / W;
    uint64_t gy = outer < 65535 ? outer : 65535;
    uint64_t chunks = 1;
    const uint64_t have = tiles * gy;
    if (have < col_blocks && len > 64) {
      chunks = col_blocks / have;                           // whole waves: no half-empty last wave
      if (chunks < 1) chunks = 1;
      const uint64_t max_chunks = (len + 63) / 64;          // >= 64 rows per chunk
      if (chunks > max_chunks) chunks = max_chunks;
      if (chunks > 65535) chunks = 65535;
    }
    const uint64_t cl = len ? (len + chunks - 1) / chunks : 1;   // len 0: one empty chunk
    chunks = len ? (len + cl - 1) / cl : 1;
    p.chunks = (uint32_t)chunks;
    p.chunk_len = cl;
    p.grid = dim3((unsigned)tiles, (unsigned)gy, (unsigned)chunks);
  } else {
    p.kind = 2;
    p.chunks = 1;
    p.chunk_len = len;
    p.grid = dim3(grid_for(outer * inner, 256), 1, 1);
  }
  return p;
}

// resident blocks per SM of the (ungated) column kernel, VEC 1 or 4; -1 if unknown
template <int OP>
int cols_occupancy(bool vec) {
  static int cols_occ[2] = {0, 0};                        // per instantiation: VEC 1 / 4
  const int vi = vec ? 1 : 0;
  if (cols_occ[vi] == 0) {
    int b = 0;
    const cudaError_t e =
        vi ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_reduce_cols<OP, 4, COL_PLAIN>, kRedThreads, 0)
           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_reduce_cols<OP, 1, COL_PLAIN>, kRedThreads, 0);
    cols_occ[vi] = (e == cudaSuccess && b > 0) ? b : -1;
    cudaGetLastError();
  }
  return cols_occ[vi];
}

// Blocks of k_fold_chunks_xchg that are resident at once (every block waits
// for the peers' puts): at most the SMs times its occupancy, the header block
// included.
template <int OP>
unsigned xchg_fold_blocks(uint64_t nout) {
  static int occ = 0;
  if (occ == 0) {
    int b = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_fold_chunks_xchg<OP>, 256, 0);
    occ = (e == cudaSuccess && b > 0) ? b : 1;
    cudaGetLastError();
  }
  const uint64_t cap = (uint64_t)dev_info().sm_count * (uint64_t)occ - 1;
  const uint64_t need = (nout + 31) / 32;
  return (unsigned)(need < cap ? need : cap) + 1;             // + the header block
}

// The exchange a sharded axis reduction's last stage runs (null: none).
struct XchgFold {
  const PeerXfer* p = nullptr;
  uint64_t len_total = 0;
  RedOut fin;                 // the final outputs
  bool* done = nullptr;       // set when the last stage exchanged and folded
};

template <int OP>
cudaError_t run_reduce(const float* x, uint64_t outer, uint64_t len, uint64_t inner, uint64_t so, uint64_t sl,
                       uint64_t si, const RedOut& ro, void* ws, size_t ws_bytes, cudaStream_t st,
                       const XchgFold& xf = XchgFold{}) {
  if (outer == 0 || inner == 0) return cudaSuccess;
  if (len == 0) return cudaErrorInvalidValue;
  Plan p = make_plan(outer, len, inner, so, sl, si, x);
  if (p.kind == 1) {
    const int occ = cols_occupancy<OP>(p.vec);
    if (occ > 0) p = make_plan(outer, len, inner, so, sl, si, x, occ);
  }
  unsigned long long* part = (unsigned long long*)ws;
  const uint32_t nparts = p.chunks;
  if (nparts > 1) {
    const size_t need = (size_t)outer * inner * nparts * sizeof(unsigned long long);
    if (!ws || ws_bytes < need) return cudaErrorInvalidValue;
  }
  if (p.kind == 0) {
    if (p.vec) launch_pdl(k_reduce_rows<OP, true>, dim3(p.grid), dim3(kRedThreads), 0, st, x, outer, len, so, p.chunks, p.chunk_len, ro, part);
    else launch_pdl(k_reduce_rows<OP, false>, dim3(p.grid), dim3(kRedThreads), 0, st, x, outer, len, so, p.chunks, p.chunk_len, ro, part);
  } else if (p.kind == 3) {
    if (p.vec) launch_pdl(k_reduce_rows_block<OP, true>, dim3(p.grid), dim3(kRedThreads), 0, st, x, outer, len, so, ro);
    else launch_pdl(k_reduce_rows_block<OP, false>, dim3(p.grid), dim3(kRedThreads), 0, st, x, outer, len, so, ro);
  } else if (p.kind == 1) {
    if (p.vec) launch_pdl(k_reduce_cols<OP, 4, COL_PLAIN>, dim3(p.grid), dim3(kRedThreads), 0, st, x, outer, len, inner, so, sl, p.chunks, p.chunk_len, ro, part, ColXform{});
    else launch_pdl(k_reduce_cols<OP, 1, COL_PLAIN>, dim3(p.grid), dim3(kRedThreads), 0, st, x, outer, len, inner, so, sl, p.chunks, p.chunk_len, ro, part, ColXform{});
  } else {
    launch_pdl(k_reduce_generic<OP>, dim3(p.grid), dim3(256), 0, st, x, outer, len, inner, so, sl, si, ro);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || nparts == 1) return e;
  const uint64_t nout = outer * inner;
  if (xf.p) {
    if (xf.done) *xf.done = true;
    return launch_pdl(k_fold_chunks_xchg<OP>, dim3(xchg_fold_blocks<OP>(nout)), dim3(256), 0, st,
                      (const unsigned long long*)part, nout, nparts, inner, xf.len_total, ro.idx_off, xf.fin, *xf.p);
  }
  return launch_pdl(k_fold_chunks<OP>, dim3(grid_for(nout, 32)), dim3(256), 0, st, (const unsigned long long*)part,
                    nout, nparts, inner, len, ro);
}

cudaError_t dispatch_reduce(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner, uint64_t so,
                            uint64_t sl, uint64_t si, const RedOut& ro, void* ws, size_t ws_bytes, cudaStream_t st,
                            const XchgFold& xf = XchgFold{}) {
  switch (op) {
    case RED_SUM: return run_reduce<RED_SUM>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    case RED_MEAN: return run_reduce<RED_MEAN>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    case RED_MAX: return run_reduce<RED_MAX>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    case RED_ARGMAX: return run_reduce<RED_ARGMAX>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    case RED_MIN: return run_reduce<RED_MIN>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    case RED_ARGMIN: return run_reduce<RED_ARGMIN>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    case RED_SUMSQ: return run_reduce<RED_SUMSQ>(x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st, xf);
    default: return cudaErrorInvalidValue;
  }
}

// identity partials (a shard with nothing to reduce)
template <int OP>
__global__ void k_identity_packed(unsigned long long* packed, uint64_t n) {
  pdl_entry();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += stride)
    packed[k] = Acc<OP>::identity_pack();
}

template <int OP>
cudaError_t run_fold_packed(const unsigned long long* parts, uint32_t nparts, uint64_t nout, uint64_t stride,
                            uint64_t len_total, const RedOut& ro, cudaStream_t st) {
  // parts[p * stride + k]: the chunk-fold layout with outer = 1, inner = stride
  // (k < nout <= stride, so the fold's outer index is always 0); launched as a
  // programmatic dependent of the kernel that produced the parts
  return launch_pdl(k_fold_chunks<OP>, dim3(grid_for(nout, 32)), dim3(256), 0, st, parts, nout, nparts, stride,
                    len_total, ro);
}

}  // namespace

size_t reduce_strided_ws_bytes(uint64_t outer, uint64_t len, uint64_t inner, uint64_t so, uint64_t sl,
                               uint64_t si) {
  // the plan depends on pointer alignment only through the vector choice;
  // size for the larger of the two plans (an empty axis or output needs none)
  if (len == 0 || outer == 0 || inner == 0) return 0;
  size_t best = 0;
  const float* probes[2] = {nullptr, reinterpret_cast<const float*>(4)};
  for (const float* pr : probes) {
    Plan p = make_plan(outer, len, inner, so, sl, si, pr);
    const uint64_t nparts = p.chunks;
    if (nparts > 1) {
      size_t b = (size_t)outer * inner * nparts * sizeof(unsigned long long);
      if (b > best) best = b;
    }
  }
  return best;
}

cudaError_t launch_reduce_strided(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                                  uint64_t so, uint64_t sl, uint64_t si, float* out, int32_t* out_idx, void* ws,
                                  size_t ws_bytes, cudaStream_t st) {
  RedOut ro;
  ro.out = out;
  ro.idx = out_idx;
  return dispatch_reduce(op, x, outer, len, inner, so, sl, si, ro, ws, ws_bytes, st);
}

size_t relu_grad_colsum_ws_bytes(uint64_t rows, uint64_t cols) {
  return reduce_strided_ws_bytes(1, rows, cols, 0, cols, 1);
}

namespace {
// A column sum fused with the elementwise pass that produces its input (see
// ColMode): bias_grad's column plan over the transformed [rows, cols] matrix,
// made for the pointer bias_grad would read (`out`), so the same chunks and the
// same sums as the two dispatches.  acc (optional): acc += the sums (grad_accum).
template <int MODE>
cudaError_t launch_xform_colsum(const float* x, const float* aux, float* out, float* db, float* acc, uint64_t rows,
                                uint64_t cols, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (cols == 0) return cudaSuccess;
  if (rows == 0) return cudaMemsetAsync(db, 0, cols * sizeof(float), st);   // acc + 0 = acc
  Plan p = make_plan(1, rows, cols, 0, cols, 1, out);
  const int occ = cols_occupancy<RED_SUM>(p.vec);
  if (occ > 0) p = make_plan(1, rows, cols, 0, cols, 1, out, occ);
  // 128-bit accesses need every operand aligned; the chunking stays the plan's
  const bool vec = p.vec && aligned16_h(x) && aligned16_h(aux);
  unsigned long long* part = (unsigned long long*)ws;
  if (p.chunks > 1) {
    const size_t need = (size_t)cols * p.chunks * sizeof(unsigned long long);
    if (!ws || ws_bytes < need) return cudaErrorInvalidValue;
  }
  RedOut ro;
  ro.out = db;
  ro.acc = acc;
  ColXform xf;
  xf.aux = aux;
  xf.out = out;
  if (vec) {
    launch_pdl(k_reduce_cols<RED_SUM, 4, MODE>, dim3(p.grid), dim3(kRedThreads), 0, st, x, (uint64_t)1, rows, cols,
               (uint64_t)0, cols, p.chunks, p.chunk_len, ro, part, xf);
  } else {
    const dim3 grid((unsigned)((cols + 31) / 32), 1, p.grid.z);       // scalar tiles are 32 columns wide
    launch_pdl(k_reduce_cols<RED_SUM, 1, MODE>, grid, dim3(kRedThreads), 0, st, x, (uint64_t)1, rows, cols,
               (uint64_t)0, cols, p.chunks, p.chunk_len, ro, part, xf);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.chunks == 1) return e;
  return launch_pdl(k_fold_chunks<RED_SUM>, dim3(grid_for(cols, 32)), dim3(256), 0, st,
                    (const unsigned long long*)part, cols, p.chunks, cols, rows, ro);
}
}  // namespace

cudaError_t launch_relu_grad_colsum(const float* g, const float* y, float* dx, float* db, uint64_t rows,
                                    uint64_t cols, void* ws, size_t ws_bytes, cudaStream_t st, float* acc) {
  return launch_xform_colsum<COL_RELU_GRAD>(g, y, dx, db, acc, rows, cols, ws, ws_bytes, st);
}

cudaError_t launch_bias_relu_colsum(const float* x, const float* b, float* y, float* col, uint64_t rows,
                                    uint64_t cols, void* ws, size_t ws_bytes, cudaStream_t st) {
  return launch_xform_colsum<COL_BIAS_RELU>(x, b, y, col, nullptr, rows, cols, ws, ws_bytes, st);
}

size_t reduce3d_ws_bytes(int op, uint64_t outer, uint64_t len, uint64_t inner) {
  (void)op;
  if (inner == 1) return reduce_strided_ws_bytes(outer, len, 1, len, 1, 1);
  return reduce_strided_ws_bytes(outer, len, inner, len * inner, inner, 1);
}

cudaError_t launch_reduce3d(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner, float* out,
                            int32_t* out_idx, void* ws, cudaStream_t st) {
  const size_t need = reduce3d_ws_bytes(op, outer, len, inner);
  RedOut ro;
  ro.out = out;
  ro.idx = out_idx;
  if (inner == 1) return dispatch_reduce(op, x, outer, len, 1, len, 1, 1, ro, ws, need, st);
  return dispatch_reduce(op, x, outer, len, inner, len * inner, inner, 1, ro, ws, need, st);
}

cudaError_t launch_reduce3d_packed(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                                   int32_t idx_off, unsigned long long* packed, void* ws, cudaStream_t st) {
  RedOut ro;
  ro.packed = packed;
  ro.idx_off = idx_off;
  const uint64_t nout = outer * inner;
  if (nout == 0) return cudaSuccess;
  if (len == 0) {
    const unsigned b = grid_for(nout, 256);
    switch (op) {
      case RED_SUM: launch_pdl(k_identity_packed<RED_SUM>, dim3(b), dim3(256), 0, st, packed, nout); break;
      case RED_MEAN: launch_pdl(k_identity_packed<RED_MEAN>, dim3(b), dim3(256), 0, st, packed, nout); break;
      case RED_MAX: launch_pdl(k_identity_packed<RED_MAX>, dim3(b), dim3(256), 0, st, packed, nout); break;
      case RED_ARGMAX: launch_pdl(k_identity_packed<RED_ARGMAX>, dim3(b), dim3(256), 0, st, packed, nout); break;
      case RED_MIN: launch_pdl(k_identity_packed<RED_MIN>, dim3(b), dim3(256), 0, st, packed, nout); break;
      case RED_ARGMIN: launch_pdl(k_identity_packed<RED_ARGMIN>, dim3(b), dim3(256), 0, st, packed, nout); break;
      case RED_SUMSQ: launch_pdl(k_identity_packed<RED_SUMSQ>, dim3(b), dim3(256), 0, st, packed, nout); break;
      default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  const size_t need = reduce3d_ws_bytes(op, outer, len, inner);
  if (inner == 1) return dispatch_reduce(op, x, outer, len, 1, len, 1, 1, ro, ws, need, st);
  return dispatch_reduce(op, x, outer, len, inner, len * inner, inner, 1, ro, ws, need, st);
}

namespace {
// The rank fold of a sharded axis reduction, in the same launch as the exchange
// over peer memory (dct_peer.cuh): every block stores its slice of the staged
// record, then thread k of the folding blocks folds output k over the ranks'
// packed partials in rank order as each arrives (ties to the lower index; mean
// divides by len_total).  The grid's last block folds nothing: it waits for
// every peer's last word (the slot reuse ordering) and checks that the shards
// tile the axis, off the folding blocks' path.
template <int OP>
__global__ void __launch_bounds__(256) k_peer_fold_axis(const __grid_constant__ PeerXfer p, uint64_t nout,
                                                        uint64_t len_total, RedOut ro) {
  pdl_entry();                                         // the record comes from the previous kernel
  bool gave_up = false;
  peer_put(p);
  const unsigned fold_grid = gridDim.x - 1;
  if (blockIdx.x == fold_grid) {
    peer_sync(p, gave_up, true);
    peer_check_axis(p, gave_up, true);
    return;
  }
  if (!ro.out && !ro.idx) return;                      // an invalid rank only takes part in the exchange
  const uint64_t step = (uint64_t)fold_grid * blockDim.x;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nout; k += step) {
    Acc<OP> a;
    a.reset();
    for (int r = 0; r < p.world; ++r) {
      Acc<OP> t;
      t.unpack(peer_get(p, r, k, gave_up));
      a.merge(t);
    }
    a.emit(ro, k, len_total);
  }
}
}  // namespace

cudaError_t launch_peer_fold_axis(int op, const PeerXfer& p, unsigned blocks, uint64_t nout, uint64_t len_total,
                                  float* out, int32_t* out_idx, cudaStream_t st) {
  blocks += 1;                                           // + the check block
  RedOut ro;
  ro.out = out;
  ro.idx = out_idx;
  switch (op) {
    case RED_SUM: launch_pdl(k_peer_fold_axis<RED_SUM>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    case RED_MEAN: launch_pdl(k_peer_fold_axis<RED_MEAN>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    case RED_MAX: launch_pdl(k_peer_fold_axis<RED_MAX>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    case RED_ARGMAX: launch_pdl(k_peer_fold_axis<RED_ARGMAX>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    case RED_MIN: launch_pdl(k_peer_fold_axis<RED_MIN>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    case RED_ARGMIN: launch_pdl(k_peer_fold_axis<RED_ARGMIN>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    case RED_SUMSQ: launch_pdl(k_peer_fold_axis<RED_SUMSQ>, dim3(blocks), dim3(256), 0, st, p, nout, len_total, ro); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_reduce3d_xchg(int op, const float* x, uint64_t outer, uint64_t len, uint64_t inner,
                                 int32_t idx_off, const PeerXfer& p, uint64_t len_total, float* out,
                                 int32_t* out_idx, void* ws, unsigned fold_blocks, cudaStream_t st) {
  const uint64_t nout = outer * inner;
  if (nout == 0) return cudaSuccess;
  unsigned long long* rec = const_cast<unsigned long long*>(p.rec);
  bool done = false;
  cudaError_t e;
  if (len == 0) {
    e = launch_reduce3d_packed(op, x, outer, len, inner, idx_off, rec, ws, st);     // identity partials
  } else {
    RedOut ro;
    ro.packed = rec;                    // a single-chunk plan emits the record here
    ro.idx_off = idx_off;
    XchgFold xf;
    xf.p = &p;
    xf.len_total = len_total;
    xf.fin.out = out;
    xf.fin.idx = out_idx;
    xf.done = &done;
    const size_t need = reduce3d_ws_bytes(op, outer, len, inner);
    e = inner == 1 ? dispatch_reduce(op, x, outer, len, 1, len, 1, 1, ro, ws, need, st, xf)
                   : dispatch_reduce(op, x, outer, len, inner, len * inner, inner, 1, ro, ws, need, st, xf);
  }
  if (e != cudaSuccess || done) return e;
  return launch_peer_fold_axis(op, p, fold_blocks, nout, len_total, out, out_idx, st);
}

cudaError_t launch_fold_packed(int op, const unsigned long long* parts, uint32_t nparts, uint64_t nout,
                               uint64_t stride, uint64_t len_total, float* out, int32_t* out_idx, cudaStream_t st) {
  if (nout == 0) return cudaSuccess;
  if (stride < nout) return cudaErrorInvalidValue;
  RedOut ro;
  ro.out = out;
  ro.idx = out_idx;
  switch (op) {
    case RED_SUM: return run_fold_packed<RED_SUM>(parts, nparts, nout, stride, len_total, ro, st);
    case RED_MEAN: return run_fold_packed<RED_MEAN>(parts, nparts, nout, stride, len_total, ro, st);
    case RED_MAX: return run_fold_packed<RED_MAX>(parts, nparts, nout, stride, len_total, ro, st);
    case RED_ARGMAX: return run_fold_packed<RED_ARGMAX>(parts, nparts, nout, stride, len_total, ro, st);
    case RED_MIN: return run_fold_packed<RED_MIN>(parts, nparts, nout, stride, len_total, ro, st);
    case RED_ARGMIN: return run_fold_packed<RED_ARGMIN>(parts, nparts, nout, stride, len_total, ro, st);
    case RED_SUMSQ: return run_fold_packed<RED_SUMSQ>(parts, nparts, nout, stride, len_total, ro, st);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// broadcast gradient (sum over the dims an operand was broadcast along)
// ---------------------------------------------------------------------------
namespace {

// Collapsed view of g: alternating groups of kept / reduced dims.
struct SumPlan {
  int ng = 0;
  uint64_t ext[kSumMaxDims];
  bool red[kSumMaxDims];
};

SumPlan plan_sum(int ndim, const int64_t* gshape, const int64_t* tshape) {
  SumPlan p;
  for (int d = 0; d < ndim; ++d) {
    const uint64_t e = (uint64_t)gshape[d];
    if (e == 1) continue;                                   // carries nothing
    const bool r = tshape[d] == 1;
    if (p.ng > 0 && p.red[p.ng - 1] == r) { p.ext[p.ng - 1] *= e; continue; }
    p.ext[p.ng] = e;
    p.red[p.ng] = r;
    ++p.ng;
  }
  return p;
}

// Generic form (two or more reduced groups): one thread per output element and
// chunk of the reduced index space, walked with an odometer; fp64 sums, folded
// over chunks in a fixed order by k_fold_chunks.
struct SumMap {
  int nk, nr;
  uint64_t kext[kSumMaxDims];
  uint64_t kstr[kSumMaxDims];
  uint64_t rext[kSumMaxDims];
  uint64_t rstr[kSumMaxDims];
};

__global__ void __launch_bounds__(256) k_sum_generic(const float* __restrict__ g, SumMap m, uint64_t nout,
                                                     uint64_t rtot, uint64_t cl, float* out,
                                                     unsigned long long* part) {
  pdl_entry();
  const uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= nout) return;
  uint64_t rem = k, base = 0;
  for (int i = m.nk - 1; i >= 0; --i) {
    const uint64_t q = rem / m.kext[i];
    base += (rem - q * m.kext[i]) * m.kstr[i];
    rem = q;
  }
  const uint64_t r0 = (uint64_t)blockIdx.y * cl;
  const uint64_t r1 = min(rtot, r0 + cl);
  uint64_t ridx[kSumMaxDims];
  uint64_t off = 0;
  rem = r0;
  for (int j = m.nr - 1; j >= 0; --j) {
    const uint64_t q = rem / m.rext[j];
    ridx[j] = rem - q * m.rext[j];
    off += ridx[j] * m.rstr[j];
    rem = q;
  }
  double s = 0.0;
  for (uint64_t r = r0; r < r1; ++r) {
    s += (double)g[base + off];
    for (int j = m.nr - 1; j >= 0; --j) {                   // odometer step, last group fastest
      off += m.rstr[j];
      if (++ridx[j] < m.rext[j]) break;
      off -= m.rstr[j] * m.rext[j];
      ridx[j] = 0;
    }
  }
  if (gridDim.y == 1) out[k] = (float)s;
  else part[(uint64_t)blockIdx.y * nout + k] = (unsigned long long)__double_as_longlong(s);
}

struct GenericSplit {
  uint64_t nout, rtot, chunks, cl;
};

GenericSplit split_generic(const SumPlan& p) {
  GenericSplit s{1, 1, 1, 1};
  for (int i = 0; i < p.ng; ++i) (p.red[i] ? s.rtot : s.nout) *= p.ext[i];
  const DevInfo& d = dev_info();
  const uint64_t target = (uint64_t)d.sm_count * d.max_threads_per_sm * 2;
  if (s.nout < target && s.rtot > 256) {
    s.chunks = std::min<uint64_t>((target + s.nout - 1) / s.nout, (s.rtot + 255) / 256);
    s.chunks = std::min<uint64_t>(s.chunks, 65535);
  }
  s.cl = (s.rtot + s.chunks - 1) / s.chunks;
  s.chunks = (s.rtot + s.cl - 1) / s.cl;
  return s;
}

}  // namespace

size_t sum_to_shape_ws_bytes(int ndim, const int64_t* gshape, const int64_t* tshape) {
  if (ndim < 0 || ndim > kSumMaxDims) return 0;
  const SumPlan p = plan_sum(ndim, gshape, tshape);
  int nred = 0;
  for (int i = 0; i < p.ng; ++i) nred += p.red[i];
  if (nred == 0) return 0;
  if (nred == 1 && p.ng <= 3) {                             // [K][R][K]: one 3-D reduction
    uint64_t o = 1, l = 1, in = 1;
    int i = 0;
    if (!p.red[0]) o = p.ext[i++];
    l = p.ext[i++];
    if (i < p.ng) in = p.ext[i];
    return reduce3d_ws_bytes(RED_SUM, o, l, in);
  }
  const GenericSplit s = split_generic(p);
  return s.chunks > 1 ? (size_t)(s.nout * s.chunks * sizeof(unsigned long long)) : 0;
}

cudaError_t launch_sum_to_shape(const float* g, int ndim, const int64_t* gshape, const int64_t* tshape,
                                float* out, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (ndim < 0 || ndim > kSumMaxDims) return cudaErrorInvalidValue;
  uint64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    if (gshape[d] < 0 || !(tshape[d] == 1 || tshape[d] == gshape[d])) return cudaErrorInvalidValue;
    n *= (uint64_t)gshape[d];
  }
  const SumPlan p = plan_sum(ndim, gshape, tshape);
  uint64_t nout = 1;
  int nred = 0;
  for (int i = 0; i < p.ng; ++i) {
    if (p.red[i]) ++nred;
    else nout *= p.ext[i];
  }
  if (n == 0) {                                             // empty input: sums of nothing
    uint64_t tn = 1;
    for (int d = 0; d < ndim; ++d) tn *= (uint64_t)tshape[d];
    return tn ? cudaMemsetAsync(out, 0, tn * sizeof(float), st) : cudaSuccess;
  }
  if (nred == 0) return cudaMemcpyAsync(out, g, n * sizeof(float), cudaMemcpyDeviceToDevice, st);
  if (nred == 1 && p.ng <= 3) {
    uint64_t o = 1, l = 1, in = 1;
    int i = 0;
    if (!p.red[0]) o = p.ext[i++];
    l = p.ext[i++];
    if (i < p.ng) in = p.ext[i];
    return launch_reduce3d(RED_SUM, g, o, l, in, out, nullptr, ws, st);
  }
  // generic: strides of each group in g (row-major, contiguous)
  SumMap m{};
  uint64_t stride = 1;
  uint64_t gstr[kSumMaxDims];
  for (int i = p.ng - 1; i >= 0; --i) { gstr[i] = stride; stride *= p.ext[i]; }
  for (int i = 0; i < p.ng; ++i) {
    if (p.red[i]) { m.rext[m.nr] = p.ext[i]; m.rstr[m.nr] = gstr[i]; ++m.nr; }
    else { m.kext[m.nk] = p.ext[i]; m.kstr[m.nk] = gstr[i]; ++m.nk; }
  }
  const GenericSplit sp = split_generic(p);
  unsigned long long* part = (unsigned long long*)ws;
  if (sp.chunks > 1 && (!ws || ws_bytes < sp.nout * sp.chunks * sizeof(unsigned long long)))
    return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((sp.nout + 255) / 256), (unsigned)sp.chunks, 1);
  if (grid.x == 0 || (sp.nout + 255) / 256 > 0x7fffffffull) return cudaErrorInvalidValue;
  launch_pdl(k_sum_generic, dim3(grid), dim3(256), 0, st, g, m, sp.nout, sp.rtot, sp.cl, out, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || sp.chunks == 1) return e;
  return launch_fold_packed(RED_SUM, part, (uint32_t)sp.chunks, sp.nout, sp.nout, sp.rtot, out, nullptr, st);
}

// ---------------------------------------------------------------------------
// full reductions: pass 1 -> one fp64 (or val/idx) partial per block,
// pass 2 -> one block folds the partials in block order.
// ---------------------------------------------------------------------------
constexpr int kFullThreads = 512;

size_t full_reduce_ws_bytes() {
  const DevInfo& d = dev_info();
  return (size_t)d.sm_count * (d.max_threads_per_sm / kFullThreads) * 2 * sizeof(double) + 256;
}

template <int OP>
__global__ void __launch_bounds__(kFullThreads) k_full_pass1(const float* __restrict__ x, uint64_t n, double* part) {
  pdl_entry();
  __shared__ double sh[32];
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double acc = 0.0;
  float mx = (OP == RED_MAX) ? -INFINITY : INFINITY;
  bool nan = false;
  const bool vec = aligned16(x);
  auto take = [&](float v) {
    if constexpr (OP == RED_SUM) acc += (double)v;
    else if constexpr (OP == RED_SUMSQ) { double d = (double)v; acc += d * d; }
    else if constexpr (OP == RED_MAX) { if (isnan(v)) nan = true; else mx = fmaxf(mx, v); }
    else { if (isnan(v)) nan = true; else mx = fminf(mx, v); }
  };
  if (vec) {
    const uint64_t n4 = n >> 2;
    uint64_t i = tid;
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = ld_stream4(x + 4 * (i + k * stride));
#pragma unroll
      for (int k = 0; k < 4; ++k) { take(v[k].x); take(v[k].y); take(v[k].z); take(v[k].w); }
    }
    for (; i < n4; i += stride) { float4 v = ld_stream4(x + 4 * i); take(v.x); take(v.y); take(v.z); take(v.w); }
    const uint64_t t = 4 * n4 + tid;
    if (t < n) take(x[t]);
  } else {
    for (uint64_t i = tid; i < n; i += stride) take(x[i]);
  }
  if constexpr (OP == RED_MAX || OP == RED_MIN) {
    // encode as double: NaN wins, else the extreme
    acc = nan ? (double)NAN : (double)mx;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      double ov = __shfl_down_sync(0xffffffffu, acc, o);
      if (isnan(ov) || (!isnan(acc) && ((OP == RED_MAX) ? ov > acc : ov < acc))) acc = ov;
    }
    if (lane == 0) sh[wid] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = sh[0];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
        double ov = sh[w];
        if (isnan(ov) || (!isnan(t) && ((OP == RED_MAX) ? ov > t : ov < t))) t = ov;
      }
      part[blockIdx.x] = t;
    }
  } else {
    double t = block_sum(acc, sh);
    if (threadIdx.x == 0) part[blockIdx.x] = t;
  }
}

// The block's fold of the pass-1 partials; the result is thread 0's.
template <int OP>
DCT_DEV double full_pass2_value(const double* part, int nparts, double* sh) {
  if constexpr (OP == RED_MAX || OP == RED_MIN) {
    double t = 0.0;
    if (threadIdx.x == 0) {
      t = part[0];
      for (int k = 1; k < nparts; ++k) {
        double ov = part[k];
        if (isnan(ov) || (!isnan(t) && ((OP == RED_MAX) ? ov > t : ov < t))) t = ov;
      }
    }
    return t;
  } else {
    // fixed assignment: thread t sums parts t, t+B, ... in order, then block tree
    const double acc = strided_sum(part, nparts);
    return block_sum(acc, sh);
  }
}

template <int OP>
__global__ void k_full_pass2(const double* part, int nparts, uint64_t n, int post, float* out32, double* out64) {
  pdl_entry();
  __shared__ double sh[32];
  double t = full_pass2_value<OP>(part, nparts, sh);
  if (threadIdx.x == 0) {
    if (post == 1) t = t / (double)n;                 // mean
    else if (post == 2) t = sqrt(t / (double)n);      // rms
    out32[0] = (float)t;
    if (out64) out64[0] = t;
  }
}

// Pass 2 of a sharded full reduction, in the same launch as the exchange over
// peer memory: thread 0 stores this rank's value (record word 0) into every
// peer's slot, block 0 the header [count, valid, -], and thread 0 folds every
// rank's record in rank order (fold_full; post 1 divides by the global count).
template <int OP>
__global__ void k_full_pass2_xchg(const double* part, int nparts, int post, float* out32, double* out64,
                                  const __grid_constant__ PeerXfer p) {
  pdl_entry();
  __shared__ double sh[32];
  bool gave_up = false;
  peer_put_header(p);
  const double t = full_pass2_value<OP>(part, nparts, sh);
  if (threadIdx.x == 0) {
    peer_put_word(p, 0, (unsigned long long)__double_as_longlong(t));
    fold_full(PeerRecsOwn0{p, gave_up, t}, p.world, OP, post, out32, out64, p.err);
  }
  peer_sync(p, gave_up);
}

static cudaError_t full_reduce_post(int op, const float* x, uint64_t n, float* out32, double* out64, void* ws,
                                    int post, cudaStream_t st) {
  if (!ws) return cudaErrorInvalidValue;
  double* part = (double*)ws;
  const DevInfo& d = dev_info();
  const int maxb = d.sm_count * (d.max_threads_per_sm / kFullThreads);
  uint64_t need = (n + 4 * (uint64_t)kFullThreads - 1) / (4 * (uint64_t)kFullThreads);
  int blocks = (int)(need < (uint64_t)maxb ? need : (uint64_t)maxb);
  if (blocks < 1) blocks = 1;
  switch (op) {
    case RED_SUM: launch_pdl(k_full_pass1<RED_SUM>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2<RED_SUM>, dim3(1), dim3(1024), 0, st, part, blocks, n, post, out32, out64); break;
    case RED_SUMSQ: launch_pdl(k_full_pass1<RED_SUMSQ>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2<RED_SUMSQ>, dim3(1), dim3(1024), 0, st, part, blocks, n, post, out32, out64); break;
    case RED_MAX: launch_pdl(k_full_pass1<RED_MAX>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2<RED_MAX>, dim3(1), dim3(32), 0, st, part, blocks, n, 0, out32, out64); break;
    case RED_MIN: launch_pdl(k_full_pass1<RED_MIN>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2<RED_MIN>, dim3(1), dim3(32), 0, st, part, blocks, n, 0, out32, out64); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_full_reduce_xchg(int op, const float* x, uint64_t n, const PeerXfer& p, int post, float* out32,
                                    double* out64, void* ws, cudaStream_t st) {
  if (!ws || n == 0) return cudaErrorInvalidValue;
  double* part = (double*)ws;
  const DevInfo& d = dev_info();
  const int maxb = d.sm_count * (d.max_threads_per_sm / kFullThreads);
  uint64_t need = (n + 4 * (uint64_t)kFullThreads - 1) / (4 * (uint64_t)kFullThreads);
  int blocks = (int)(need < (uint64_t)maxb ? need : (uint64_t)maxb);
  if (blocks < 1) blocks = 1;
  switch (op) {
    case RED_SUM: launch_pdl(k_full_pass1<RED_SUM>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2_xchg<RED_SUM>, dim3(1), dim3(1024), 0, st, part, blocks, post, out32, out64, p); break;
    case RED_SUMSQ: launch_pdl(k_full_pass1<RED_SUMSQ>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2_xchg<RED_SUMSQ>, dim3(1), dim3(1024), 0, st, part, blocks, post, out32, out64, p); break;
    case RED_MAX: launch_pdl(k_full_pass1<RED_MAX>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2_xchg<RED_MAX>, dim3(1), dim3(32), 0, st, part, blocks, post, out32, out64, p); break;
    case RED_MIN: launch_pdl(k_full_pass1<RED_MIN>, dim3(blocks), dim3(kFullThreads), 0, st, x, n, part);
      launch_pdl(k_full_pass2_xchg<RED_MIN>, dim3(1), dim3(32), 0, st, part, blocks, post, out32, out64, p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_full_reduce(int op, const float* x, uint64_t n, float* out32, double* out64, void* ws,
                               cudaStream_t st) {
  if (n == 0) {
    // the sum of nothing is 0 and its mean NaN (all-ones bytes are a NaN in
    // both widths); max / min have no identity
    if (op == RED_SUM || op == RED_SUMSQ || op == RED_MEAN) {
      const int byte = op == RED_MEAN ? 0xFF : 0;
      cudaError_t e = cudaMemsetAsync(out32, byte, sizeof(float), st);
      if (e == cudaSuccess && out64) e = cudaMemsetAsync(out64, byte, sizeof(double), st);
      return e;
    }
    return cudaErrorInvalidValue;
  }
  if (op == RED_MEAN) return full_reduce_post(RED_SUM, x, n, out32, out64, ws, 1, st);
  return full_reduce_post(op, x, n, out32, out64, ws, 0, st);
}

cudaError_t launch_rms(const float* x, uint64_t n, float* out, void* ws, cudaStream_t st) {
  if (n == 0) return cudaMemsetAsync(out, 0, sizeof(float), st);
  return full_reduce_post(RED_SUMSQ, x, n, out, nullptr, ws, 2, st);
}

// ---------------------------------------------------------------------------
// grad_sq_reduce / grad_norm_final (the reference's two-pass clip)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_grad_sq(const float* __restrict__ g, uint64_t count, float* part, uint64_t off,
                                                 uint64_t ngroups) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t grp = gw; grp < ngroups; grp += nw) {
    double acc = 0.0;
    const uint64_t b = grp * 256;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint64_t i = b + (uint64_t)k * 32 + lane;
      if (i < count) { double d = (double)g[i]; acc += d * d; }
    }
    acc = warp_sum(acc);
    if (lane == 0) part[off + grp] = (float)acc;
  }
}

cudaError_t launch_grad_sq_reduce(const float* g, uint64_t count, float* partials, uint64_t off, uint64_t ngroups,
                                  cudaStream_t st) {
  if (ngroups == 0) return cudaSuccess;
  const uint64_t threads = ngroups * 32;
  launch_pdl(k_grad_sq, dim3(grid_for(threads, 256)), dim3(256), 0, st, g, count, partials, off, ngroups);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(1024) k_grad_norm_final(const float* part, uint64_t n, float max_norm, float* ns) {
  pdl_entry();
  __shared__ double sh[32];
  double t = block_sum(strided_sum(part, n), sh);
  if (threadIdx.x == 0) {
    const float norm = (float)sqrt(t);
    ns[0] = norm;
    ns[1] = norm > max_norm ? (float)((double)max_norm / ((double)norm + (double)1e-6f)) : 1.0f;
  }
}

cudaError_t launch_grad_norm_final(const float* partials, uint64_t n, float max_norm, float* ns, cudaStream_t st) {
  launch_pdl(k_grad_norm_final, dim3(1), dim3(1024), 0, st, partials, n, max_norm, ns);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// dice sums (nn_dice_loss_sums.hlsl:19-55, nn_dice_loss.hlsl:19-53): per
// sample (sum p*t, sum p, sum t) in float64.  Block (b, c) streams chunk c of
// sample b -- float4 loads when the samples are 16-byte aligned -- and leaves
// three float64 partials; one warp per sample folds them in chunk order
// (lane-strided, then a fixed shuffle tree), so the sums are the same on every
// run.  A sample of one chunk is written by its block directly.
// ---------------------------------------------------------------------------
namespace {
constexpr int kDiceThreads = 256;

DCT_DEV void dice_emit(double si, double sp, double st, float* out, uint64_t b, int mode) {
  if (mode == 0) {
    out[b * 3 + 0] = (float)si;
    out[b * 3 + 1] = (float)sp;
    out[b * 3 + 2] = (float)st;
  } else {
    out[b] = (float)(1.0 - 2.0 * si / (sp + st + (double)1e-6f));
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kDiceThreads) k_dice_partials(const float* __restrict__ pred,
                                                                const float* __restrict__ target, uint32_t size,
                                                                uint32_t chunks, uint32_t chunk_len, double* part,
                                                                float* out, int mode) {
  pdl_entry();
  __shared__ double sh[32];
  const uint64_t b = blockIdx.x / chunks;
  const uint32_t c = blockIdx.x - (uint32_t)b * chunks;
  const uint64_t base = b * size;
  const uint32_t l0 = c * chunk_len, l1 = min(size, l0 + chunk_len);
  double si = 0.0, sp = 0.0, st = 0.0;
  if (VEC) {                                    // size, chunk_len and the bases are float4 multiples
    // 4 float4 pairs in flight per thread, loads first, then the adds in index order
    constexpr int U = 4;
    uint32_t i = l0 + 4 * threadIdx.x;
    for (; i + 4 * kDiceThreads * (U - 1) < l1; i += 4 * kDiceThreads * U) {
      float4 p[U], t[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        p[k] = ld_stream4(pred + base + i + 4 * kDiceThreads * k);
        t[k] = ld_stream4(target + base + i + 4 * kDiceThreads * k);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        si += (double)p[k].x * (double)t[k].x; sp += (double)p[k].x; st += (double)t[k].x;
        si += (double)p[k].y * (double)t[k].y; sp += (double)p[k].y; st += (double)t[k].y;
        si += (double)p[k].z * (double)t[k].z; sp += (double)p[k].z; st += (double)t[k].z;
        si += (double)p[k].w * (double)t[k].w; sp += (double)p[k].w; st += (double)t[k].w;
      }
    }
    for (; i < l1; i += 4 * kDiceThreads) {
      const float4 p = ld_stream4(pred + base + i), t = ld_stream4(target + base + i);
      si += (double)p.x * (double)t.x; sp += (double)p.x; st += (double)t.x;
      si += (double)p.y * (double)t.y; sp += (double)p.y; st += (double)t.y;
      si += (double)p.z * (double)t.z; sp += (double)p.z; st += (double)t.z;
      si += (double)p.w * (double)t.w; sp += (double)p.w; st += (double)t.w;
    }
  } else {
    for (uint32_t i = l0 + threadIdx.x; i < l1; i += kDiceThreads) {
      const double p = (double)ld_stream(pred + base + i), t = (double)ld_stream(target + base + i);
      si += p * t; sp += p; st += t;
    }
  }
  si = block_sum(si, sh);
  __syncthreads();
  sp = block_sum(sp, sh);
  __syncthreads();
  st = block_sum(st, sh);
  if (threadIdx.x == 0) {
    if (chunks == 1) {
      dice_emit(si, sp, st, out, b, mode);
    } else {
      double* q = part + ((uint64_t)b * chunks + c) * 3;
      q[0] = si; q[1] = sp; q[2] = st;
    }
  }
}

__global__ void __launch_bounds__(256) k_dice_fold(const double* __restrict__ part, uint32_t batch, uint32_t chunks,
                                                   float* out, int mode) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const uint64_t b = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (b >= batch) return;
  double si = 0.0, sp = 0.0, st = 0.0;
  for (uint32_t c = lane; c < chunks; c += 32) {
    const double* q = part + (b * chunks + c) * 3;
    si += q[0]; sp += q[1]; st += q[2];
  }
  si = warp_sum(si);
  sp = warp_sum(sp);
  st = warp_sum(st);
  if (lane == 0) dice_emit(si, sp, st, out, b, mode);
}
struct DicePlan {
  uint32_t chunks = 1, chunk_len = 0;
};

// chunks per sample: two full waves of blocks over the batch (at the partials
// kernel's own occupancy, so no partly filled last wave), >= 4096 elements a
// chunk, chunk starts on a float4 boundary
DicePlan dice_plan(uint32_t batch, uint32_t size) {
  static int occ = 0;
  if (occ == 0) {
    int b = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_dice_partials<true>, kDiceThreads, 0);
    occ = (e == cudaSuccess && b > 0) ? b : dev_info().max_threads_per_sm / kDiceThreads;
    cudaGetLastError();
  }
  DicePlan p;
  const uint64_t want = (uint64_t)dev_info().sm_count * (uint64_t)occ * 2;
  uint64_t chunks = batch ? want / batch : 1;                  // rounded down: at most the two waves
  const uint64_t max_chunks = ((uint64_t)size + 4095) / 4096;
  if (chunks > max_chunks) chunks = max_chunks;
  if (chunks < 1) chunks = 1;
  uint64_t cl = ((uint64_t)size + chunks - 1) / chunks;
  cl = (cl + 3) & ~3ull;
  if (cl == 0) cl = 4;
  p.chunks = (uint32_t)(size ? ((uint64_t)size + cl - 1) / cl : 1);
  p.chunk_len = (uint32_t)cl;
  return p;
}
}  // namespace

size_t dice_ws_bytes(uint32_t batch, uint32_t size) {
  const DicePlan p = dice_plan(batch, size);
  return p.chunks > 1 ? (size_t)batch * p.chunks * 3 * sizeof(double) : 0;
}

cudaError_t launch_dice_sums(const float* pred, const float* target, uint32_t batch, uint32_t size, float* out,
                             int mode, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (batch == 0) return cudaSuccess;
  const DicePlan p = dice_plan(batch, size);
  if (p.chunks > 1 && (!ws || ws_bytes < dice_ws_bytes(batch, size))) return cudaErrorInvalidValue;
  const bool vec = size % 4 == 0 && aligned16_h(pred) && aligned16_h(target);
  const unsigned blocks = (unsigned)((uint64_t)batch * p.chunks);
  double* part = (double*)ws;
  if (vec) launch_pdl(k_dice_partials<true>, dim3(blocks), dim3(kDiceThreads), 0, st, pred, target, size, p.chunks,
                      p.chunk_len, part, out, mode);
  else launch_pdl(k_dice_partials<false>, dim3(blocks), dim3(kDiceThreads), 0, st, pred, target, size, p.chunks,
                  p.chunk_len, part, out, mode);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.chunks == 1) return e;
  launch_pdl(k_dice_fold, dim3((unsigned)(((uint64_t)batch * 32 + 255) / 256)), dim3(256), 0, st,
             (const double*)part, batch, p.chunks, out, mode);
  return cudaGetLastError();
}

}  // namespace dct
