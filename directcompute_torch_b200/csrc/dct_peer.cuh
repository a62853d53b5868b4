// The record exchange over NVLink peer memory, as device code shared by the
// kernels that fold the exchanged records (dist.cu: full sums, the softmax-CE
// loss, BatchNorm channel sums; k_reduce.cu: axis reductions).
//
// Each rank stores its record straight into every rank's slot (plain 16-byte
// stores to a peer's memory mapped with CUDA IPC), fences at system scope and
// release-stores the exchange's epoch into that rank's flag for it.  Every block
// of the folding kernel then waits, bounded by %globaltimer, until every rank's
// flag here holds the epoch, acquires each flag in every thread, and folds its
// share of the local slots -- put, wait and fold in one launch.  No load ever
// reads another GPU's memory.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "dct_common.cuh"

namespace dct {

// The host-known part of a record: n u64 words (bit patterns) at offset `off`.
struct Hdr {
  uint32_t off = 0, n = 0;
  unsigned long long v[4] = {0, 0, 0, 0};
};

struct PeerXfer {
  const unsigned long long* rec;     // this rank's record, words [0, h.off)
  Hdr h;                             // and its header words
  void* const* bases;                // every rank's exchange region (mapped here)
  uint64_t slot_off, flag_off;       // this rank's slot / flag in every region
  unsigned long long epoch;
  const unsigned long long* flags;   // this rank's flags of this parity, one per rank
  int world;
  unsigned long long timeout_ns;
  uint32_t* err;
  const unsigned long long* slots;   // this rank's slots of this parity: rank r's record at r * stride
  uint64_t stride;
  int64_t axis_nout;                 // >= 0: axis records; block 0 checks that the shards tile the axis
};

// Block q < world stores the record into rank q's slot and raises rank q's flag;
// then every block waits for all flags (bounded: past the deadline the error
// word gets DCT_DEVERR_PEER_WAIT and the block goes on) and every thread
// acquires them.  Ends with the block synchronised.
DCT_DEV void peer_put_wait(const PeerXfer& p) {
  if ((int)blockIdx.x < p.world) {
    unsigned char* base = static_cast<unsigned char*>(p.bases[blockIdx.x]);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(base + p.slot_off);
    const uint64_t n = p.h.off;
    const uint64_t n2 = n >> 1;
    const uint4* s4 = reinterpret_cast<const uint4*>(p.rec);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (uint64_t i = threadIdx.x; i < n2; i += blockDim.x) d4[i] = s4[i];
    if ((n & 1) && threadIdx.x == 0) dst[n - 1] = p.rec[n - 1];
    if (threadIdx.x < p.h.n) dst[n + threadIdx.x] = p.h.v[threadIdx.x];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long* flag = reinterpret_cast<unsigned long long*>(base + p.flag_off);
      asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(p.epoch) : "memory");
    }
  }
  for (int q = threadIdx.x; q < p.world; q += blockDim.x) {
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p.flags + q) : "memory");
      if (v >= p.epoch) break;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > p.timeout_ns) {
        if (p.err) atomicOr(p.err, DCT_DEVERR_PEER_WAIT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  for (int q = 0; q < p.world; ++q) {               // every thread's own acquire of every record
    [[maybe_unused]] unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p.flags + q) : "memory");
  }
  // axis-reduction records: the shards must tile [0, len_total) in rank order
  if (p.axis_nout >= 0 && blockIdx.x == 0 && threadIdx.x == 0) {
    const uint64_t nout = (uint64_t)p.axis_nout;
    unsigned long long expect = 0, total = p.slots[nout + 2];
    bool ok = true;
    for (int r = 0; r < p.world; ++r) {
      const unsigned long long* hh = p.slots + (uint64_t)r * p.stride + nout;
      ok &= (hh[3] == 1ull) && (hh[0] == expect) && (hh[2] == total);
      expect += hh[1];
    }
    ok &= (expect == total);
    if (!ok && p.err) atomicOr(p.err, DCT_DEVERR_PEER_INVALID);
  }
}

}  // namespace dct
