// Rank-order folds of the exchanged records of the sharded ops, and the
// readers they fold through: records gathered by NCCL into local memory, or
// the tagged lines of the peer exchange (dct_peer.cuh).  The kernels that fold
// after a separate exchange (dist.cu) and the producing kernels that run the
// exchange themselves (k_reduce.cu, k_softmax.cu, k_batchnorm.cu) share them,
// so both transports give the same bits.
#pragma once
#include <math.h>

#include "dct_common.cuh"
#include "dct_peer.cuh"
#include "kernels.h"

namespace dct {

// Record readers for the folds: word i of rank r as a double.  LocalRecs
// reads the records an NCCL all-gather left in local memory; PeerRecs reads
// them over the peer exchange (dct_peer.cuh), this rank's from its record.
struct LocalRecs {
  const double* all;
  uint64_t stride;
  DCT_DEV double operator()(int r, uint64_t i) const { return all[(uint64_t)r * stride + i]; }
};
struct PeerRecs {
  const PeerXfer& p;
  bool& gave_up;
  DCT_DEV double operator()(int r, uint64_t i) const { return peer_get_f64(p, r, i, gave_up); }
};
// The same, with this rank's word 0 held in a register by the kernel that
// computed it (its header words still come from p.h).
struct PeerRecsOwn0 {
  const PeerXfer& p;
  bool& gave_up;
  double own0;
  DCT_DEV double operator()(int r, uint64_t i) const {
    return (r == p.rank && i == 0) ? own0 : peer_get_f64(p, r, i, gave_up);
  }
};

// Full reduction records [value, count, valid, -]: fold in rank order.
// post: 0 none, 1 mean (divide by the total count).  One thread.
template <class G>
DCT_DEV void fold_full(const G& get, int world, int op, int post, float* out32, double* out64, uint32_t* err) {
  double acc = 0.0, cnt = 0.0;
  bool ok = true, first = true;
  const bool ext = (op == RED_MAX || op == RED_MIN);
  for (int r = 0; r < world; ++r) {
    const double n = get(r, 1);
    ok &= (get(r, 2) == 1.0);
    cnt += n;
    if (ext) {
      if (n == 0.0) continue;                            // empty shard: no candidate
      const double v = get(r, 0);
      if (first || isnan(v) || (!isnan(acc) && (op == RED_MAX ? v > acc : v < acc))) acc = v;
      first = false;
    } else {
      const double v = get(r, 0);
      acc = first ? v : acc + v;
      first = false;
    }
  }
  if (ext && first) ok = false;                          // max / min of nothing
  if (post == 1) acc = acc / cnt;
  if (!ok) {
    acc = (double)NAN;
    if (err) atomicOr(err, DCT_DEVERR_PEER_INVALID);
  }
  if (out32) out32[0] = (float)acc;
  if (out64) out64[0] = acc;
}

// Softmax-CE records [sum of row losses, rows, valid, -] -> loss = sum / div.  One thread.
template <class G>
DCT_DEV void fold_loss(const G& get, int world, double div, float* loss, uint32_t* err) {
  double acc = 0.0;
  bool ok = true;
  for (int r = 0; r < world; ++r) {
    ok &= (get(r, 2) == 1.0);
    const double v = get(r, 0);
    acc = r == 0 ? v : acc + v;
  }
  if (!ok && err) atomicOr(err, DCT_DEVERR_PEER_INVALID);
  if (loss) loss[0] = ok ? (float)(acc / div) : NAN;
}

// Channel-sum records [nsum sums][count, valid, nsum, -]: out[j] = sum over
// ranks in rank order; out[nsum] = total count.  Item j of nsum + 1.
template <class G>
DCT_DEV void fold_sums(const G& get, int world, uint32_t nsum, double* out, uint32_t* err, uint32_t j) {
  if (j < nsum) {
    double acc = get(0, j);
    for (int r = 1; r < world; ++r) acc += get(r, j);
    out[j] = acc;
  } else if (j == nsum) {
    double cnt = 0.0;
    bool ok = true;
    for (int r = 0; r < world; ++r) {
      cnt += get(r, nsum);
      ok &= (get(r, nsum + 1) == 1.0) && (get(r, nsum + 2) == (double)nsum);
    }
    out[nsum] = cnt;
    if (!ok && err) atomicOr(err, DCT_DEVERR_PEER_INVALID);
  }
}

}  // namespace dct
