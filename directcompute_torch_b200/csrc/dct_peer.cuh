// The record exchange over NVLink peer memory, as device code shared by the
// kernels that fold the exchanged records (dist.cu: full sums, the softmax-CE
// loss, BatchNorm channel sums; k_reduce.cu: axis reductions).
//
// A record is a run of 64-bit words.  Each word crosses NVLink as two 64-bit
// lines, its low and its high 32 bits each paired with the exchange's 32-bit
// tag, in one 16-byte store of two single-copy-atomic 64-bit elements.  Every
// block of the folding kernel first stores a slice of this rank's record into
// every peer's slot; the folding threads then read the peers' lines they need
// from their own GPU's memory, spinning (bounded by %globaltimer) until both
// lines of a word carry this exchange's tag.  A line proves its own arrival,
// so there are no fences and no flags: put, wait and fold are one launch, and
// no load ever reads another GPU's memory.  This rank's own words come straight
// from its record.
//
// Slots alternate by exchange parity.  Block 0 of every fold reads one line of
// every peer (peer_sync), so a rank's fold of exchange e + 1 ends only after
// every peer has stored its e + 1 lines, which each peer does only after its
// own fold of e has ended (stream order).  A rank therefore stores e + 2 into a
// peer's parity slot only after that peer has read the e lines there.  Tags
// run 1, 2, ..., 2^32 - 1, 1, ... in zeroed slots: a line left from exchange
// e - 2 or never written never carries the tag of e.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "dct_common.cuh"

namespace dct {

// The peer exchange serves at most this many ranks (the axis check stages
// every rank's header in shared memory); larger worlds use NCCL.
constexpr int kPeerMaxWorld = 64;

// The host-known part of a record: n u64 words (bit patterns) at offset `off`.
struct Hdr {
  uint32_t off = 0, n = 0;
  unsigned long long v[4] = {0, 0, 0, 0};
};

struct PeerXfer {
  const unsigned long long* rec;     // this rank's record, words [0, h.off)
  Hdr h;                             // and its header words [h.off, h.off + h.n)
  void* const* bases;                // every rank's exchange region (mapped here)
  uint64_t slot_off;                 // byte offset of this rank's slot (this parity) in every region
  uint32_t tag;                      // this exchange's tag, never 0
  int rank, world;
  unsigned long long timeout_ns;
  uint32_t* err;
  const unsigned long long* slots;   // this rank's slots of this parity: rank r's lines at r * stride
  uint64_t stride;                   // lines per rank slot
  int64_t axis_nout;                 // >= 0: axis records; block 0 checks that the shards tile the axis
};

DCT_DEV uint64_t peer_words(const PeerXfer& p) { return (uint64_t)p.h.off + p.h.n; }

DCT_DEV unsigned long long peer_word(const PeerXfer& p, uint64_t i) {
  return i < p.h.off ? p.rec[i] : p.h.v[i - p.h.off];
}

// Word i of this rank's record, value w, into every peer's slot.
DCT_DEV void peer_put_word(const PeerXfer& p, uint64_t i, unsigned long long w) {
  const unsigned long long tag = (unsigned long long)p.tag << 32;
  const unsigned long long lo = (w & 0xffffffffull) | tag, hi = (w >> 32) | tag;
  for (int q = 0; q < p.world; ++q) {
    if (q == p.rank) continue;
    unsigned long long* dst =
        reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(p.bases[q]) + p.slot_off) + 2 * i;
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(lo), "l"(hi) : "memory");
  }
}

// Every block stores its slice of this rank's record (record words then header
// words) into every peer's slot.
DCT_DEV void peer_put(const PeerXfer& p) {
  const uint64_t nw = peer_words(p);
  const uint64_t per = (nw + gridDim.x - 1) / gridDim.x;
  const uint64_t w0 = (uint64_t)blockIdx.x * per, w1 = min(nw, w0 + per);
  for (uint64_t i = w0 + threadIdx.x; i < w1; i += blockDim.x) peer_put_word(p, i, peer_word(p, i));
}

// The designated block (block 0 unless the kernel names another) stores the
// header words (a kernel that puts its record words itself).
DCT_DEV void peer_put_header(const PeerXfer& p, bool mine) {
  if (mine && threadIdx.x < p.h.n) peer_put_word(p, p.h.off + threadIdx.x, p.h.v[threadIdx.x]);
}
DCT_DEV void peer_put_header(const PeerXfer& p) { peer_put_header(p, blockIdx.x == 0); }

// Word i of rank r's record: this rank's from its record, a peer's once both of
// its lines carry this exchange's tag.  `gave_up` is the calling thread's:
// after one wait runs out (the error word gets DCT_DEVERR_PEER_WAIT) the thread
// waits no more and reads whatever is there.
DCT_DEV unsigned long long peer_get(const PeerXfer& p, int r, uint64_t i, bool& gave_up) {
  if (r == p.rank) return peer_word(p, i);
  const unsigned long long* src = p.slots + (uint64_t)r * p.stride + 2 * i;
  unsigned long long lo, hi, t0 = 0;
  bool started = false;
  for (;;) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "l"(src) : "memory");
    if (((uint32_t)(lo >> 32) == p.tag && (uint32_t)(hi >> 32) == p.tag) || gave_up) break;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (!started) {
      t0 = t;
      started = true;
    } else if (t - t0 > p.timeout_ns) {
      if (p.err) atomicOr(p.err, DCT_DEVERR_PEER_WAIT);
      gave_up = true;
      break;
    }
  }
  return (lo & 0xffffffffull) | (hi << 32);
}

DCT_DEV double peer_get_f64(const PeerXfer& p, int r, uint64_t i, bool& gave_up) {
  return __longlong_as_double((long long)peer_get(p, r, i, gave_up));
}

// The designated block: thread q waits for peer q's last word (the ordering the
// slot reuse relies on, whatever the fold itself reads).
DCT_DEV void peer_sync(const PeerXfer& p, bool& gave_up, bool mine) {
  if (!mine) return;
  for (int q = threadIdx.x; q < p.world; q += blockDim.x)
    if (q != p.rank) (void)peer_get(p, q, peer_words(p) - 1, gave_up);
}
DCT_DEV void peer_sync(const PeerXfer& p, bool& gave_up) { peer_sync(p, gave_up, blockIdx.x == 0); }

// The designated block of an axis reduction (every thread of that block calls
// it): the shards' headers [offset, len, len_total, valid] must tile
// [0, len_total) in rank order.  The block fetches every rank's four header
// words at once.
DCT_DEV void peer_check_axis(const PeerXfer& p, bool& gave_up, bool mine) {
  if (p.axis_nout < 0 || !mine) return;
  __shared__ unsigned long long hv[kPeerMaxWorld][4];
  const uint64_t nout = (uint64_t)p.axis_nout;
  for (int t = threadIdx.x; t < 4 * p.world; t += blockDim.x) hv[t >> 2][t & 3] = peer_get(p, t >> 2, nout + (t & 3), gave_up);
  __syncthreads();
  if (threadIdx.x != 0) return;
  unsigned long long expect = 0;
  const unsigned long long total = hv[0][2];
  bool ok = true;
  for (int r = 0; r < p.world; ++r) {
    ok &= (hv[r][3] == 1ull) && (hv[r][0] == expect) && (hv[r][2] == total);
    expect += hv[r][1];
  }
  ok &= (expect == total);
  if (!ok && p.err) atomicOr(p.err, DCT_DEVERR_PEER_INVALID);
}
DCT_DEV void peer_check_axis(const PeerXfer& p, bool& gave_up) { peer_check_axis(p, gave_up, blockIdx.x == 0); }

// The start of every fold kernel over peer memory: put, then the ordering wait
// and (axis records) the shard check.
DCT_DEV void peer_begin(const PeerXfer& p, bool& gave_up) {
  peer_put(p);
  peer_sync(p, gave_up);
  peer_check_axis(p, gave_up);
}

}  // namespace dct
