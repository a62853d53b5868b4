// Sharding layer of libdct_cuda: one process per GPU, NCCL over NVLink/NVSwitch.
//
// The reference drives a single D3D11 device and has no multi-GPU path
// (engine.cpp:61-129 creates one device and one immediate context).  These
// dct_dist_* entry points are the data-parallel extension of its hot path.
// Each rank holds one contiguous shard of the sharded axis (rows of C2/C3/C4,
// the batch N of C5b, a flat slice of C5a), and the ops whose result depends on
// other shards make exactly one exchange:
//
//   axis reduction over the sharded axis   one packed 8-byte partial per output
//   full reduction                          (float64 value, count)
//   softmax-CE loss                         (float64 sum of row losses, rows)
//   BatchNorm statistics / backward sums    C x 2 float64 channel sums + count
//
// Every exchange is one ncclAllGather of fixed-size records into a [world]
// array, folded on the device in rank order: results are identical on every
// rank and from run to run, and at world size 1 bit-identical to the
// single-GPU entry points.  Each record ends with a header (shard offset,
// count, validity); a rank whose arguments are bad still takes part with an
// invalid header, so all ranks take the same collective steps and all of them
// report the failure (DCT_ERR_DIST at the next wait) instead of hanging.
//
// NCCL is loaded with dlopen (DCT_NCCL_LIB, else an already-loaded
// libnccl.so.2, else the loader's libnccl.so.2), so the library loads and runs
// single-GPU work where NCCL is absent.  Init is bounded by the deadline given
// to dct_dist_init (ranks that never join end in an error, not a hang).  While
// a communicator is active every wait of the library polls the stream, the
// communicator's asynchronous error and the deadline, and aborts the
// communicator on failure (a peer that died cannot hang this process).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <memory>
#include <initializer_list>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "dct_common.cuh"
#include "dct_fold.cuh"
#include "kernels.h"
#include "runtime_internal.h"
#include "../../include/dct_cuda.h"

namespace dct {
namespace {

struct NcclApi {
  void* h = nullptr;
  int version = 0;
  decltype(&ncclGetVersion) GetVersion = nullptr;
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRank) CommInitRank = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommFinalize) CommFinalize = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclAllGather) AllGather = nullptr;
  decltype(&ncclAllReduce) AllReduce = nullptr;
  decltype(&ncclBroadcast) Broadcast = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
  decltype(&ncclGetLastError) GetLastError = nullptr;
};

struct InitJob {
  std::mutex m;
  std::condition_variable cv;
  bool done = false, abandoned = false;
  ncclResult_t r = ncclSuccess;
  ncclComm_t comm = nullptr;
};

struct DistState {
  NcclApi api;
  std::string load_error;
  ncclComm_t comm = nullptr;
  int world = 0, rank = -1;
  double timeout_s = 120.0;
  bool aborted = false;
  // exchange buffers (device, stream-ordered)
  void* send = nullptr;
  size_t send_bytes = 0;
  void* recv = nullptr;
  size_t recv_bytes = 0;
  double* fold = nullptr;          // folded sums / counts (float64)
  size_t fold_bytes = 0;
  // peer-memory exchange: this rank's region holds slots [2][world][slot_bytes]
  // (by exchange parity, then by writing rank) of tagged 64-bit lines, two per
  // record word; every rank's region is mapped here (CUDA IPC over NVLink)
  bool peer = false;
  void* region = nullptr;
  size_t slot_bytes = 0;
  std::vector<void*> peer_base;
  void** peer_dev = nullptr;
  uint64_t epoch = 0;
};
DistState D;

#define DLOCK std::lock_guard<std::recursive_mutex> _dlk(rt_mutex())

template <class F>
bool sym(F& f, const char* name) {
  f = reinterpret_cast<F>(dlsym(D.api.h, name));
  return f != nullptr;
}

bool load_nccl() {
  if (D.api.h) return true;
  void* h = nullptr;
  const char* env = getenv("DCT_NCCL_LIB");
  if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    const char* e = dlerror();
    D.load_error = std::string("NCCL not found (set DCT_NCCL_LIB): ") + (e ? e : "");
    return false;
  }
  D.api.h = h;
  bool ok = sym(D.api.GetVersion, "ncclGetVersion") && sym(D.api.GetUniqueId, "ncclGetUniqueId") &&
            sym(D.api.CommInitRank, "ncclCommInitRank") && sym(D.api.CommGetAsyncError, "ncclCommGetAsyncError") &&
            sym(D.api.CommAbort, "ncclCommAbort") && sym(D.api.CommDestroy, "ncclCommDestroy") &&
            sym(D.api.AllGather, "ncclAllGather") && sym(D.api.AllReduce, "ncclAllReduce") &&
            sym(D.api.Broadcast, "ncclBroadcast") && sym(D.api.GetErrorString, "ncclGetErrorString");
  sym(D.api.CommFinalize, "ncclCommFinalize");
  sym(D.api.GetLastError, "ncclGetLastError");
  if (!ok) {
    D.load_error = "the NCCL library lacks a required symbol";
    dlclose(h);
    D.api = NcclApi{};
    return false;
  }
  D.api.GetVersion(&D.api.version);
  return true;
}

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void fail(const char* where, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void fail(const char* where, const char* fmt, ...) {
  char body[384], msg[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(body, sizeof(body), fmt, ap);
  va_end(ap);
  snprintf(msg, sizeof(msg), "%s: %s", where, body);
  note_error(DCT_ERR_DIST, msg);
}

void abort_comm() {
  if (D.comm) D.api.CommAbort(D.comm);
  D.comm = nullptr;
  D.aborted = true;
  D.peer = false;                // the mappings are released by dct_dist_finalize
  rt_dist_hooks() = DistHooks{};
}

const char* nccl_msg(ncclResult_t r) {
  static thread_local char buf[320];
  const char* last = (D.comm && D.api.GetLastError) ? D.api.GetLastError(D.comm) : "";
  snprintf(buf, sizeof(buf), "%s%s%s", D.api.GetErrorString(r), last && *last ? " / " : "", last ? last : "");
  return buf;
}

// Bring an NCCL call on `comm` to completion of its enqueue (non-blocking
// communicators answer ncclInProgress); on failure or past the deadline abort
// the library's communicator.
bool settle_on(ncclComm_t comm, ncclResult_t r, const char* where) {
  if (r == ncclSuccess) return true;
  if (r == ncclInProgress && comm) {
    const double t0 = now_s();
    for (;;) {
      ncclResult_t st = ncclSuccess;
      D.api.CommGetAsyncError(comm, &st);
      if (st == ncclSuccess) return true;
      if (st != ncclInProgress) { r = st; break; }
      const double el = now_s() - t0;
      if (el > D.timeout_s) {
        fail(where, "NCCL did not complete within %.0f s; communicator aborted", D.timeout_s);
        abort_comm();
        return false;
      }
      // an enqueue normally completes within microseconds: poll hot first, then back off
      if (el < 2e-3) std::this_thread::yield();
      else std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  fail(where, "NCCL error: %s; communicator aborted", nccl_msg(r));
  abort_comm();
  return false;
}
bool settle(ncclResult_t r, const char* where) { return settle_on(D.comm, r, where); }

bool hook_async_error(char* msg, int len) {
  if (!D.comm) return false;
  ncclResult_t st = ncclSuccess;
  if (D.api.CommGetAsyncError(D.comm, &st) != ncclSuccess) return false;
  if (st == ncclSuccess || st == ncclInProgress) return false;
  snprintf(msg, len, "%s", nccl_msg(st));
  return true;
}
void hook_abort() { abort_comm(); }

bool need_comm(const char* where) {
  if (D.comm) return true;
  fail(where, "%s", D.aborted ? "the communicator was aborted after a failure; dct_dist_finalize, then dct_dist_init"
                              : "no communicator (call dct_dist_init)");
  return false;
}

bool grow(void*& p, size_t& have, size_t want, const char* where) {
  if (have >= want) return true;
  cudaStream_t st = rt_stream();
  if (p) cudaFreeAsync(p, st);
  p = nullptr;
  have = 0;
  want = (want + 255) & ~size_t(255);
  if (!rt_cuda_ok(cudaMallocAsync(&p, want, st), where)) return false;
  have = want;
  return true;
}

bool buffers(size_t send, size_t recv, size_t fold, const char* where) {
  return grow(D.send, D.send_bytes, send, where) && grow(D.recv, D.recv_bytes, recv, where) &&
         grow(reinterpret_cast<void*&>(D.fold), D.fold_bytes, fold, where);
}

bool all_gather(const void* send, void* recv, size_t count_u64, const char* where) {
  return settle(D.api.AllGather(send, recv, count_u64, ncclUint64, D.comm, rt_stream()), where);
}

// ---------------------------------------------------------------------------
// peer-memory exchange
// ---------------------------------------------------------------------------
// Each rank stores its record straight into every peer's slot over NVLink
// (stores to a peer's memory mapped with CUDA IPC) as tagged lines, and each
// rank folds the lines in its own memory once they carry the exchange's tag
// (dct_peer.cuh).  A slot holds 32K record words (16 bytes of lines per
// word); larger records go over NCCL.
constexpr size_t kSlotBytes = 512 * 1024;

size_t slot_off(int par, int q) { return ((size_t)par * D.world + q) * D.slot_bytes; }

__global__ void k_check_axis_shards(const unsigned long long* all, int world, uint64_t stride, uint64_t nout,
                                    uint32_t* err);

unsigned long long f64_bits(double d) {
  unsigned long long u;
  memcpy(&u, &d, sizeof(u));
  return u;
}
Hdr make_hdr(uint32_t off, std::initializer_list<unsigned long long> v) {
  Hdr h;
  h.off = off;
  for (unsigned long long x : v) h.v[h.n++] = x;
  return h;
}

// header words written into a local record (the NCCL path)
__global__ void k_put_u64(unsigned long long* rec, Hdr h) {
  if (threadIdx.x < h.n) rec[h.off + threadIdx.x] = h.v[threadIdx.x];
}

// Gather every rank's record: the device part rec[0, h.off) plus the header
// words h.  Over peer memory nothing is launched here: *px describes the put
// and the wait, which the caller's fold kernel runs itself (dct_peer.cuh), and
// the function returns XCH_PEER.  Over NCCL the all-gather runs now, *all =
// the records (record q at *all + q * *stride), and it returns XCH_NCCL; the
// caller folds with a separate kernel.  axis_nout >= 0 also checks
// axis-reduction shard headers (at word axis_nout of each record).  XCH_FAIL:
// the error is recorded.
enum Xch { XCH_FAIL = 0, XCH_NCCL = 1, XCH_PEER = 2 };
// whether a record of `words` words goes over peer memory
bool peer_fits(size_t words) { return D.peer && words * 16 <= D.slot_bytes; }
Xch exchange(void* rec, const Hdr& h, const unsigned long long** all, size_t* stride, PeerXfer* px,
             const char* where, int64_t axis_nout = -1) {
  cudaStream_t st = rt_stream();
  const size_t n = (size_t)h.off + h.n;
  if (peer_fits(n)) {
    const unsigned long long ep = ++D.epoch;
    const int par = (int)(ep & 1);
    unsigned char* base = static_cast<unsigned char*>(D.region);
    const unsigned long long* slots = reinterpret_cast<const unsigned long long*>(base + slot_off(par, 0));
    // the device gives up at 0.8 of the host's deadline, so its error (a peer's
    // record did not arrive) reaches the host before the host's own deadline
    const double lim = 0.8 * (D.timeout_s < 30.0 ? D.timeout_s : 30.0);
    px->rec = static_cast<const unsigned long long*>(rec);
    px->h = h;
    px->bases = (void* const*)D.peer_dev;
    px->slot_off = (uint64_t)slot_off(par, D.rank);
    px->tag = (uint32_t)((ep - 1) % 0xffffffffull) + 1u;
    px->rank = D.rank;
    px->world = D.world;
    px->timeout_ns = (unsigned long long)(lim * 1e9);
    px->err = device_error_word();
    px->slots = slots;
    px->stride = (uint64_t)(D.slot_bytes / 8);
    px->axis_nout = axis_nout;
    *all = nullptr;
    *stride = 0;
    return XCH_PEER;
  }
  unsigned long long* r64 = static_cast<unsigned long long*>(rec);
  if (h.n) k_put_u64<<<1, 32, 0, st>>>(r64, h);
  if (!rt_cuda_ok(cudaGetLastError(), where)) return XCH_FAIL;
  if (!all_gather(rec, D.recv, n, where)) return XCH_FAIL;
  *all = static_cast<const unsigned long long*>(D.recv);
  *stride = n;
  if (axis_nout >= 0) {
    k_check_axis_shards<<<1, 32, 0, st>>>(*all, D.world, n, (uint64_t)axis_nout, device_error_word());
    if (!rt_cuda_ok(cudaGetLastError(), where)) return XCH_FAIL;
  }
  return XCH_NCCL;
}

// blocks of a put-wait-fold kernel: every rank's put block, enough to fold
// `work` items 256 at a time, never more than one per SM (all resident at once,
// since every block waits for every rank's record, its own rank's included)
unsigned fold_blocks(uint64_t work) {
  uint64_t b = (work + 255) / 256;
  const uint64_t cap = (uint64_t)std::max(D.world, dev_info().sm_count);
  if (b > cap) b = cap;
  if (b < (uint64_t)D.world) b = (uint64_t)D.world;
  return (unsigned)b;
}

void peer_teardown() {
  for (int q = 0; q < (int)D.peer_base.size(); ++q)
    if (q != D.rank && D.peer_base[q]) cudaIpcCloseMemHandle(D.peer_base[q]);
  D.peer_base.clear();
  if (D.peer_dev) cudaFree(D.peer_dev);
  if (D.region) cudaFree(D.region);
  D.peer_dev = nullptr;
  D.region = nullptr;
  D.peer = false;
  D.epoch = 0;
  cudaGetLastError();
}

// Map every rank's exchange region (all ranks or none: the outcome is agreed
// over the communicator).  DCT_PEER_EXCHANGE=0 keeps NCCL all-gathers.
bool peer_setup() {
  const char* env = getenv("DCT_PEER_EXCHANGE");
  bool ok = !(env && env[0] == '0') && D.world <= kPeerMaxWorld;
  D.slot_bytes = kSlotBytes;
  const size_t bytes = 2 * (size_t)D.world * D.slot_bytes;
  cudaIpcMemHandle_t mine{};
  if (ok) ok = cudaMalloc(&D.region, bytes) == cudaSuccess && cudaMemset(D.region, 0, bytes) == cudaSuccess &&
               cudaDeviceSynchronize() == cudaSuccess && cudaIpcGetMemHandle(&mine, D.region) == cudaSuccess;
  cudaGetLastError();
  // all ranks' handles (64 bytes each) over the communicator
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  unsigned char* dh = nullptr;
  std::vector<unsigned char> all(hb * D.world);
  bool xok = cudaMalloc(&dh, hb * (D.world + 1)) == cudaSuccess &&
             cudaMemcpy(dh, &mine, hb, cudaMemcpyHostToDevice) == cudaSuccess &&
             settle(D.api.AllGather(dh, dh + hb, hb, ncclUint8, D.comm, rt_stream()), "dct_dist_init(handles)") &&
             rt_wait_stream("dct_dist_init(handles)") &&
             cudaMemcpy(all.data(), dh + hb, hb * D.world, cudaMemcpyDeviceToHost) == cudaSuccess;
  if (dh) cudaFree(dh);
  cudaGetLastError();
  if (!xok) { peer_teardown(); return false; }      // the communicator itself failed
  D.peer_base.assign(D.world, nullptr);
  if (ok) {
    D.peer_base[D.rank] = D.region;
    for (int q = 0; q < D.world && ok; ++q) {
      if (q == D.rank) continue;
      cudaIpcMemHandle_t h;
      memcpy(&h, all.data() + hb * q, hb);
      ok = cudaIpcOpenMemHandle(&D.peer_base[q], h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    }
    if (ok) ok = cudaMalloc(&D.peer_dev, sizeof(void*) * D.world) == cudaSuccess &&
                 cudaMemcpy(D.peer_dev, D.peer_base.data(), sizeof(void*) * D.world, cudaMemcpyHostToDevice) ==
                     cudaSuccess;
    cudaGetLastError();
  }
  // agree: the peer path only if every rank mapped every region
  int* flag = nullptr;
  int agreed = 0;
  const int mine_ok = ok ? 1 : 0;
  bool aok = cudaMalloc(&flag, sizeof(int)) == cudaSuccess &&
             cudaMemcpy(flag, &mine_ok, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
             settle(D.api.AllReduce(flag, flag, 1, ncclInt32, ncclMin, D.comm, rt_stream()), "dct_dist_init(agree)") &&
             rt_wait_stream("dct_dist_init(agree)") &&
             cudaMemcpy(&agreed, flag, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
  if (flag) cudaFree(flag);
  cudaGetLastError();
  if (!aok || !agreed) {
    peer_teardown();
    return false;
  }
  D.peer = true;
  D.epoch = 0;
  return true;
}

// ---------------------------------------------------------------------------
// record headers and rank-order folds
// ---------------------------------------------------------------------------
// Shards of an axis reduction must tile [0, len_total) in rank order and agree
// on len_total; any invalid or inconsistent header marks the result invalid.
__global__ void k_check_axis_shards(const unsigned long long* all, int world, uint64_t stride, uint64_t nout,
                                    uint32_t* err) {
  if (threadIdx.x != 0) return;
  unsigned long long expect = 0, total = all[nout + 2];
  bool ok = true;
  for (int r = 0; r < world; ++r) {
    const unsigned long long* h = all + (uint64_t)r * stride + nout;
    ok &= (h[3] == 1ull) && (h[0] == expect) && (h[2] == total);
    expect += h[1];
  }
  ok &= (expect == total);
  if (!ok && err) atomicOr(err, DCT_DEVERR_PEER_INVALID);
}

// the folds after an NCCL all-gather
__global__ void k_fold_full(const double* all, uint64_t stride, int world, int op, int post, float* out32,
                            double* out64, uint32_t* err) {
  grid_dep_wait();
  if (threadIdx.x == 0) fold_full(LocalRecs{all, stride}, world, op, post, out32, out64, err);
}
__global__ void k_fold_loss(const double* all, uint64_t stride, int world, double div, float* loss, uint32_t* err) {
  grid_dep_wait();
  if (threadIdx.x == 0) fold_loss(LocalRecs{all, stride}, world, div, loss, err);
}
__global__ void k_fold_sums(const double* all, uint64_t stride, int world, uint32_t nsum, double* out,
                            uint32_t* err) {
  grid_dep_wait();
  fold_sums(LocalRecs{all, stride}, world, nsum, out, err, blockIdx.x * blockDim.x + threadIdx.x);
}

// the same folds over peer memory: put, wait and fold in one launch (dct_peer.cuh)
__global__ void __launch_bounds__(256) k_peer_fold_full(const __grid_constant__ PeerXfer p, int op, int post,
                                                        float* out32, double* out64) {
  pdl_entry();                                         // the record comes from the previous kernel
  bool gave_up = false;
  peer_begin(p, gave_up);
  if (blockIdx.x == 0 && threadIdx.x == 0) fold_full(PeerRecs{p, gave_up}, p.world, op, post, out32, out64, p.err);
}
__global__ void __launch_bounds__(256) k_peer_fold_loss(const __grid_constant__ PeerXfer p, double div,
                                                        float* loss) {
  pdl_entry();
  bool gave_up = false;
  peer_begin(p, gave_up);
  if (blockIdx.x == 0 && threadIdx.x == 0) fold_loss(PeerRecs{p, gave_up}, p.world, div, loss, p.err);
}
__global__ void __launch_bounds__(256) k_peer_fold_sums(const __grid_constant__ PeerXfer p, uint32_t nsum,
                                                        double* out) {
  pdl_entry();
  bool gave_up = false;
  peer_begin(p, gave_up);
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j <= nsum; j += gridDim.x * blockDim.x)
    fold_sums(PeerRecs{p, gave_up}, p.world, nsum, out, p.err, j);
}

Buffer* live(void* h) { return h ? rt_buf(h) : nullptr; }

}  // namespace
}  // namespace dct

using namespace dct;

extern "C" {

DCT_API int dct_dist_available(void) {
  DLOCK;
  return load_nccl() ? 1 : 0;
}

DCT_API int dct_dist_nccl_version(void) {
  DLOCK;
  return load_nccl() ? D.api.version : 0;
}

DCT_API int dct_dist_shard(uint64_t n, int world, int rank, uint64_t* offset, uint64_t* count) {
  if (world < 1 || rank < 0 || rank >= world || !offset || !count) return DCT_ERR_ARG;
  const uint64_t base = n / (uint64_t)world, rem = n % (uint64_t)world;
  const uint64_t r = (uint64_t)rank;
  *count = base + (r < rem ? 1 : 0);
  *offset = r * base + (r < rem ? r : rem);
  return 0;
}

DCT_API int dct_dist_unique_id(void* out, int len) {
  DLOCK;
  if (!out || len < (int)sizeof(ncclUniqueId)) {
    note_error(DCT_ERR_ARG, "dct_dist_unique_id: the output needs 128 bytes");
    return DCT_ERR_ARG;
  }
  if (!load_nccl()) { note_error(DCT_ERR_DIST, D.load_error.c_str()); return DCT_ERR_DIST; }
  ncclUniqueId id;
  const ncclResult_t r = D.api.GetUniqueId(&id);
  if (r != ncclSuccess) {
    fail("dct_dist_unique_id", "%s", D.api.GetErrorString(r));
    return DCT_ERR_DIST;
  }
  memcpy(out, &id, sizeof(id));
  return 0;
}

DCT_API int dct_dist_init(const void* id, int len, int nranks, int rank, double timeout_s) {
  DLOCK;
  if (!id || len < (int)sizeof(ncclUniqueId) || nranks < 1 || rank < 0 || rank >= nranks) {
    note_error(DCT_ERR_ARG, "dct_dist_init: need a 128-byte id and 0 <= rank < nranks");
    return DCT_ERR_ARG;
  }
  if (D.comm) { note_error(DCT_ERR_DIST, "dct_dist_init: already initialised (dct_dist_finalize first)"); return DCT_ERR_DIST; }
  if (!load_nccl()) { note_error(DCT_ERR_DIST, D.load_error.c_str()); return DCT_ERR_DIST; }
  if (!rt_init()) return DCT_ERR_NO_DEVICE;
  if (!rt_cuda_ok(cudaSetDevice(dev_info().device), "dct_dist_init(cudaSetDevice)")) return DCT_ERR_CUDA;
  D.timeout_s = timeout_s > 0 ? timeout_s : 120.0;
  D.aborted = false;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  // ncclCommInitRank blocks until every rank has joined.  It runs on a helper
  // thread so that this call returns DCT_ERR_DIST at the deadline when a rank
  // never joins; a helper that completes after the deadline aborts the
  // communicator it got.  (A non-blocking communicator would bound init too,
  // but costs about 35 us more host time per collective: measured on B200
  // with NCCL 2.28.)
  auto job = std::make_shared<InitJob>();
  const int dev = dev_info().device;
  const NcclApi api = D.api;
  std::thread([job, uid, nranks, rank, dev, api]() {
    cudaSetDevice(dev);
    ncclComm_t c = nullptr;
    const ncclResult_t r = api.CommInitRank(&c, nranks, uid, rank);
    std::lock_guard<std::mutex> lk(job->m);
    if (job->abandoned) {
      if (c) api.CommAbort(c);
      return;
    }
    job->r = r;
    job->comm = c;
    job->done = true;
    job->cv.notify_all();
  }).detach();
  {
    std::unique_lock<std::mutex> lk(job->m);
    const bool done = job->cv.wait_for(lk, std::chrono::duration<double>(D.timeout_s), [&] { return job->done; });
    if (!done) {
      job->abandoned = true;
      fail("dct_dist_init", "not every rank joined within %.0f s", D.timeout_s);
      return DCT_ERR_DIST;
    }
  }
  if (job->r != ncclSuccess) {
    if (job->comm) D.api.CommAbort(job->comm);
    fail("dct_dist_init", "NCCL error: %s", D.api.GetErrorString(job->r));
    return DCT_ERR_DIST;
  }
  D.comm = job->comm;
  D.world = nranks;
  D.rank = rank;
  DistHooks& hk = rt_dist_hooks();
  hk.async_error = &hook_async_error;
  hk.abort = &hook_abort;
  hk.timeout_s = D.timeout_s;
  if (!D.comm) return DCT_ERR_DIST;
  peer_setup();                                    // falls back to NCCL all-gathers when it cannot map every rank
  return D.comm ? 0 : DCT_ERR_DIST;
}

DCT_API int dct_dist_finalize(void) {
  DLOCK;
  int rc = 0;
  if (D.comm && D.peer) {
    // every rank unmaps the others' regions before any rank frees its own
    if (!rt_wait_stream("dct_dist_finalize")) rc = DCT_ERR_DIST;
    for (int q = 0; q < (int)D.peer_base.size(); ++q)
      if (q != D.rank && D.peer_base[q]) cudaIpcCloseMemHandle(D.peer_base[q]);
    for (int q = 0; q < (int)D.peer_base.size(); ++q)
      if (q != D.rank) D.peer_base[q] = nullptr;
    if (D.comm && buffers(8, 8 * (size_t)D.world, 8, "dct_dist_finalize") &&
        all_gather(D.send, D.recv, 1, "dct_dist_finalize(barrier)") && !rt_wait_stream("dct_dist_finalize"))
      rc = DCT_ERR_DIST;
    peer_teardown();
  } else if (D.aborted && !D.peer_base.empty()) {
    // After an abort no barrier is possible, and other ranks may still hold this
    // rank's region mapped: close this rank's mappings of theirs and keep its
    // own region allocated until the process exits (a later dct_dist_init makes
    // a new one).
    if (!rt_wait_stream("dct_dist_finalize")) rc = DCT_ERR_DIST;
    for (int q = 0; q < (int)D.peer_base.size(); ++q)
      if (q != D.rank && D.peer_base[q]) cudaIpcCloseMemHandle(D.peer_base[q]);
    D.peer_base.clear();
    if (D.peer_dev) cudaFree(D.peer_dev);
    D.peer_dev = nullptr;
    D.region = nullptr;
    D.epoch = 0;
    cudaGetLastError();
  }
  if (D.comm) {
    if (!rt_wait_stream("dct_dist_finalize")) rc = DCT_ERR_DIST;
    if (D.comm && D.api.CommFinalize) {
      if (!settle(D.api.CommFinalize(D.comm), "dct_dist_finalize")) rc = DCT_ERR_DIST;
    }
    if (D.comm) D.api.CommDestroy(D.comm);
  }
  D.comm = nullptr;
  rt_dist_hooks() = DistHooks{};
  D.world = 0;
  D.rank = -1;
  D.aborted = false;
  cudaStream_t st = rt_stream();
  for (void** p : {&D.send, &D.recv, reinterpret_cast<void**>(&D.fold)})
    if (*p) { cudaFreeAsync(*p, st); *p = nullptr; }
  D.send_bytes = D.recv_bytes = D.fold_bytes = 0;
  return rc;
}

DCT_API int dct_dist_rank(void) { DLOCK; return D.comm ? D.rank : -1; }
DCT_API int dct_dist_world(void) { DLOCK; return D.comm ? D.world : 0; }
DCT_API int dct_dist_peer_active(void) { DLOCK; return D.comm && D.peer ? 1 : 0; }

DCT_API int dct_dist_allreduce(void* buf, uint64_t count, int op) {
  DLOCK;
  if (!need_comm("dct_dist_allreduce")) return DCT_ERR_DIST;
  Buffer* b = live(buf);
  if (!b) { note_error(DCT_ERR_HANDLE, "dct_dist_allreduce: not a live buffer"); return DCT_ERR_HANDLE; }
  if (b->count < count) { note_error(DCT_ERR_SIZE, "dct_dist_allreduce: buffer too small"); return DCT_ERR_SIZE; }
  ncclRedOp_t o;
  switch (op) {
    case RED_SUM: o = ncclSum; break;
    case RED_MEAN: o = ncclAvg; break;
    case RED_MAX: o = ncclMax; break;
    case RED_MIN: o = ncclMin; break;
    default: note_error(DCT_ERR_ARG, "dct_dist_allreduce: op must be 0 sum, 1 mean, 2 max or 4 min"); return DCT_ERR_ARG;
  }
  return settle(D.api.AllReduce(b->d, b->d, count, ncclFloat32, o, D.comm, rt_stream()), "dct_dist_allreduce")
             ? 0 : DCT_ERR_DIST;
}

DCT_API int dct_dist_broadcast(void* buf, uint64_t count, int root) {
  DLOCK;
  if (!need_comm("dct_dist_broadcast")) return DCT_ERR_DIST;
  Buffer* b = live(buf);
  if (!b) { note_error(DCT_ERR_HANDLE, "dct_dist_broadcast: not a live buffer"); return DCT_ERR_HANDLE; }
  if (b->count < count) { note_error(DCT_ERR_SIZE, "dct_dist_broadcast: buffer too small"); return DCT_ERR_SIZE; }
  if (root < 0 || root >= D.world) { note_error(DCT_ERR_ARG, "dct_dist_broadcast: bad root"); return DCT_ERR_ARG; }
  return settle(D.api.Broadcast(b->d, b->d, count, ncclFloat32, root, D.comm, rt_stream()), "dct_dist_broadcast")
             ? 0 : DCT_ERR_DIST;
}

DCT_API int dct_dist_barrier(void) {
  DLOCK;
  if (!need_comm("dct_dist_barrier")) return DCT_ERR_DIST;
  if (!buffers(8, 8 * (size_t)D.world, 8, "dct_dist_barrier")) return DCT_ERR_CUDA;
  if (!all_gather(D.send, D.recv, 1, "dct_dist_barrier")) return DCT_ERR_DIST;
  return rt_wait_stream("dct_dist_barrier") ? 0 : DCT_ERR_DIST;
}

// x viewed as [outer, len, inner], this rank's slice [len_offset, len_offset + len)
// of a middle axis of global extent len_total; out / out_idx get the reduction
// over the whole axis on every rank.
DCT_API int dct_dist_reduce(int op, void* x, uint64_t outer, uint64_t len, uint64_t inner, uint64_t len_offset,
                            uint64_t len_total, void* out, void* out_idx) {
  DLOCK;
  const char* W = "dct_dist_reduce";
  if (!need_comm(W)) return DCT_ERR_DIST;
  if (op < RED_SUM || op > RED_SUMSQ) { note_error(DCT_ERR_ARG, "dct_dist_reduce: unknown op"); return DCT_ERR_ARG; }
  const uint64_t nout = outer * inner;
  if (nout == 0 || len_total > 0x7fffffffull) {
    note_error(DCT_ERR_ARG, "dct_dist_reduce: need outer*inner > 0 and len_total < 2^31");
    return DCT_ERR_ARG;
  }
  const uint64_t stride = nout + 4;
  if (!buffers(stride * 8, stride * 8 * (size_t)D.world, 8, W)) return DCT_ERR_CUDA;
  Buffer *bx = live(x), *bo = live(out), *bi = live(out_idx);
  const bool arg = (op == RED_ARGMAX || op == RED_ARGMIN);
  int op_run = op;                                    // max / min with indices: values and indices in one pass
  if ((op == RED_MAX || op == RED_MIN) && out_idx) op_run = op == RED_MAX ? RED_ARGMAX : RED_ARGMIN;
  bool valid = bx && (bo || (arg && bi)) && (!out_idx || bi) && bx->count >= outer * len * inner &&
               (!bo || bo->count >= nout) && (!bi || bi->count >= nout) && len_offset + len <= len_total;
  unsigned long long* send = (unsigned long long*)D.send;
  cudaStream_t st = rt_stream();
  float* o32 = bo ? bo->d : nullptr;
  int32_t* oi = bi ? reinterpret_cast<int32_t*>(bi->d) : nullptr;
  if (arg && !oi) { oi = reinterpret_cast<int32_t*>(o32); o32 = nullptr; }   // indices into out (dct_reduce rule)
  // header [offset, len, len_total, valid] after the nout packed partials
  auto hdr = [&](bool ok) { return make_hdr((uint32_t)nout, {len_offset, len, len_total, ok ? 1ull : 0ull}); };
  const unsigned long long* all = nullptr;
  size_t xs = 0;
  PeerXfer px;
  if (peer_fits(nout + 4)) {
    // Over peer memory the local reduction's last stage (the chunk fold) puts
    // this rank's partials, waits for the peers' and folds them, one launch
    // fewer than staging the record.  (Storing the partials into the peers
    // from the column kernel itself was slower: 8-byte scattered remote stores
    // from every thread of its grid.)
    if (valid && !rt_ensure_ws(reduce3d_ws_bytes(op_run, outer, len, inner))) return DCT_ERR_CUDA;
    if (exchange(send, hdr(valid), &all, &xs, &px, W, (int64_t)nout) != XCH_PEER) return DCT_ERR_DIST;
    cudaError_t e = cudaErrorInvalidValue;
    if (valid) {
      e = launch_reduce3d_xchg(op_run, bx->d, outer, len, inner, (int32_t)len_offset, px, len_total, o32, oi, rt_ws(),
                               fold_blocks(nout), st);
      if (e != cudaSuccess) cudaGetLastError();
    }
    if (e != cudaSuccess) {                          // still puts and waits: an invalid header, no outputs
      valid = false;
      px.h = hdr(false);
      e = launch_peer_fold_axis(op_run, px, fold_blocks(nout), nout, len_total, nullptr, nullptr, st);
    }
    if (!rt_cuda_ok(e, W)) return DCT_ERR_CUDA;
  } else {
    // the packed partials are staged in the local record and all-gathered
    if (valid && !rt_ensure_ws(reduce3d_ws_bytes(op_run, outer, len, inner))) return DCT_ERR_CUDA;
    if (valid && !rt_cuda_ok(launch_reduce3d_packed(op_run, bx->d, outer, len, inner, (int32_t)len_offset, send,
                                                    rt_ws(), st), W))
      valid = false;
    const Xch how = exchange(send, hdr(valid), &all, &xs, &px, W, (int64_t)nout);
    if (how == XCH_FAIL) return DCT_ERR_DIST;
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && valid) e = launch_fold_packed(op_run, all, (uint32_t)D.world, nout, xs, len_total, o32, oi, st);
    if (!rt_cuda_ok(e, W)) return DCT_ERR_CUDA;
  }
  if (!valid) { note_error(DCT_ERR_ARG, "dct_dist_reduce: invalid handles or sizes on this rank"); return DCT_ERR_ARG; }
  return 0;
}

// full reduction (0 sum, 1 mean, 2 max, 4 min, 6 sum of squares) of this
// rank's n elements, combined over all ranks into out[0] on every rank;
// *host_out64 gets the float64 value (waits) when non-null
DCT_API int dct_dist_reduce_all(int op, void* x, uint64_t n, void* out, double* host_out64) {
  DLOCK;
  const char* W = "dct_dist_reduce_all";
  if (!need_comm(W)) return DCT_ERR_DIST;
  if (!(op == RED_SUM || op == RED_MEAN || op == RED_MAX || op == RED_MIN || op == RED_SUMSQ)) {
    note_error(DCT_ERR_ARG, "dct_dist_reduce_all: op must be 0 sum, 1 mean, 2 max, 4 min or 6 sumsq");
    return DCT_ERR_ARG;
  }
  if (!buffers(32 + 8, 32 * (size_t)D.world, 16, W)) return DCT_ERR_CUDA;
  Buffer *bx = live(x), *bo = live(out);
  bool valid = bx && bo && bx->count >= n && bo->count >= 1;
  cudaStream_t st = rt_stream();
  double* rec = (double*)D.send;
  const int local_op = op == RED_MEAN ? RED_SUM : op;
  // record [value, n, valid, 0]; value = float64 sum (mean: the raw sum) or
  // extreme, computed by the reduction when one runs and 0 otherwise
  const int post = op == RED_MEAN ? 1 : 0;
  const unsigned long long hn = f64_bits((double)n);
  auto hdr = [&](bool ran, bool ok) {
    const unsigned long long hv = f64_bits(ok ? 1.0 : 0.0);
    return ran ? make_hdr(1, {hn, hv, 0ull}) : make_hdr(0, {0ull, hn, hv, 0ull});
  };
  const unsigned long long* all = nullptr;
  size_t xs = 0;
  PeerXfer px;
  if (valid && n > 0 && !rt_ensure_ws(full_reduce_ws_bytes() + 256)) return DCT_ERR_CUDA;
  cudaError_t fe = cudaSuccess;
  if (peer_fits(4)) {
    // over peer memory pass 2 of the reduction puts, waits and folds itself
    bool fused = false;
    if (valid && n > 0) {
      if (exchange(rec, hdr(true, true), &all, &xs, &px, W) != XCH_PEER) return DCT_ERR_DIST;
      fused = launch_full_reduce_xchg(local_op, bx->d, n, px, post, bo->d, D.fold, rt_ws(), st) == cudaSuccess;
      if (!fused) { cudaGetLastError(); valid = false; px.h = hdr(false, false); }
    } else if (exchange(rec, hdr(false, valid), &all, &xs, &px, W) != XCH_PEER) {
      return DCT_ERR_DIST;
    }
    if (!fused)
      fe = launch_pdl(k_peer_fold_full, dim3(fold_blocks(1)), dim3(256), 0, st, px, local_op, post,
                      valid ? bo->d : nullptr, D.fold);
  } else {
    bool ran = false;
    if (valid && n > 0) {
      float* scratch32 = reinterpret_cast<float*>(rec + 4);              // float copy of the local result, unused
      if (!rt_cuda_ok(launch_full_reduce(local_op, bx->d, n, scratch32, rec, rt_ws(), st), W)) valid = false;
      ran = valid;
    }
    if (exchange(rec, hdr(ran, valid), &all, &xs, &px, W) == XCH_FAIL) return DCT_ERR_DIST;
    fe = launch_pdl(k_fold_full, dim3(1), dim3(32), 0, st, (const double*)all, (uint64_t)xs, D.world, local_op, post,
                    valid ? bo->d : nullptr, D.fold, device_error_word());
  }
  if (!rt_cuda_ok(fe, W)) return DCT_ERR_CUDA;
  if (host_out64) {
    double* hs = rt_host_scratch();
    if (!rt_cuda_ok(cudaMemcpyAsync(hs, D.fold, 8, cudaMemcpyDeviceToHost, st), W)) return DCT_ERR_CUDA;
    if (!rt_wait_stream(W)) return DCT_ERR_DIST;
    *host_out64 = hs[0];
  }
  if (!valid) { note_error(DCT_ERR_ARG, "dct_dist_reduce_all: invalid handles or sizes on this rank"); return DCT_ERR_ARG; }
  return 0;
}

// fused softmax + CE over this rank's rows; dlogits use grad_div (the global
// batch), loss[0] = (sum of every rank's row losses) / loss_div on every rank
DCT_API int dct_dist_softmax_ce(void* logits, void* labels, int labels_int32, uint32_t rows, uint32_t K, void* probs,
                                void* dlogits, void* loss, void* logprobs, float loss_div, float grad_div) {
  DLOCK;
  const char* W = "dct_dist_softmax_ce";
  if (!need_comm(W)) return DCT_ERR_DIST;
  if (!buffers(32, 32 * (size_t)D.world, 8, W)) return DCT_ERR_CUDA;
  Buffer *bl = live(logits), *bt = live(labels), *bp = live(probs), *bd = live(dlogits), *bs = live(loss),
         *bq = live(logprobs);
  const uint64_t n = (uint64_t)rows * K;
  bool valid = bl && bl->count >= n && K > 0 && (!labels || (bt && bt->count >= rows)) &&
               (!probs || (bp && bp->count >= n)) && (!dlogits || (bd && bd->count >= n && labels)) &&
               (!loss || (bs && bs->count >= 1)) && (!logprobs || (bq && bq->count >= n));
  cudaStream_t st = rt_stream();
  double* rec = (double*)D.send;
  // record [loss sum, rows, valid, 0]; the loss sum is computed by the kernel
  // when it computes a loss and 0 otherwise
  const unsigned long long hr = f64_bits((double)rows);
  auto hdr = [&](bool ran, bool ok) {
    const unsigned long long hv = f64_bits(ok ? 1.0 : 0.0);
    return ran ? make_hdr(1, {hr, hv, 0ull}) : make_hdr(0, {0ull, hr, hv, 0ull});
  };
  const unsigned long long* all = nullptr;
  size_t xs = 0;
  PeerXfer px;
  if (valid && rows > 0 && !rt_ensure_ws(softmax_ce_ws_bytes(rows, K))) return DCT_ERR_CUDA;
  // over peer memory the loss fold puts, waits and folds itself
  const bool fuse = peer_fits(4) && valid && rows > 0 && bt;
  if (fuse && exchange(rec, hdr(true, true), &all, &xs, &px, W) != XCH_PEER) return DCT_ERR_DIST;
  bool ran = false, fused = false;
  if (valid && rows > 0) {
    SoftmaxCEArgs a;
    a.logits = bl->d;
    a.labels = bt ? bt->d : nullptr;
    a.labels_int32 = labels_int32 != 0;
    a.rows = rows;
    a.K = K;
    a.probs = bp ? bp->d : nullptr;
    a.dlogits = bd ? bd->d : nullptr;
    a.logprobs = bq ? bq->d : nullptr;
    a.grad_div = grad_div;
    a.err = device_error_word();
    if (fuse) {
      a.xchg = &px;
      a.loss = bs ? bs->d : nullptr;
      a.loss_div = (double)loss_div;
    } else {
      a.loss_partial = bt ? rec : nullptr;
    }
    if (!rt_cuda_ok(launch_softmax_ce(a, rt_ws(), st), W)) valid = false;
    ran = valid && a.loss_partial;
    fused = valid && fuse;
  }
  cudaError_t fe = cudaSuccess;
  if (fuse) {
    if (!fused) {                                   // still puts and waits: an invalid header, no loss
      px.h = hdr(false, false);
      fe = launch_pdl(k_peer_fold_loss, dim3(fold_blocks(1)), dim3(256), 0, st, px, (double)loss_div, nullptr);
    }
  } else {
    const Xch how = exchange(rec, hdr(ran, valid), &all, &xs, &px, W);
    if (how == XCH_FAIL) return DCT_ERR_DIST;
    fe = how == XCH_PEER
             ? launch_pdl(k_peer_fold_loss, dim3(fold_blocks(1)), dim3(256), 0, st, px, (double)loss_div,
                          bs && valid ? bs->d : nullptr)
             : launch_pdl(k_fold_loss, dim3(1), dim3(32), 0, st, (const double*)all, (uint64_t)xs, D.world,
                          (double)loss_div, bs && valid ? bs->d : nullptr, device_error_word());
  }
  if (!rt_cuda_ok(fe, W)) return DCT_ERR_CUDA;
  if (!valid) { note_error(DCT_ERR_ARG, "dct_dist_softmax_ce: invalid handles or sizes on this rank"); return DCT_ERR_ARG; }
  return 0;
}

namespace {
// Channel sums of this rank's x (BWD: dy, dy*x) into the send record, the
// exchange, and the rank-order fold into D.fold = [2C sums][total count].
bool bn_exchange(const float* x, const float* dy, uint32_t N, uint32_t C, uint32_t S, bool valid, const char* W,
                 int* rc) {
  const uint32_t nsum = 2 * C;
  const uint64_t stride = (uint64_t)nsum + 4;
  if (!buffers(stride * 8, stride * 8 * (size_t)D.world, ((size_t)nsum + 1) * 8, W)) { *rc = DCT_ERR_CUDA; return false; }
  cudaStream_t st = rt_stream();
  double* rec = (double*)D.send;
  if (valid && !rt_ensure_ws(bn_ws_bytes(N, C))) { *rc = DCT_ERR_CUDA; return false; }
  // header [count, valid, nsum, 0] after the 2C sums (an invalid rank's sums
  // are never used: its valid word fails the fold on every rank)
  auto hdr = [&](bool ok) {
    return make_hdr(nsum, {f64_bits((double)N * (double)S), f64_bits(ok ? 1.0 : 0.0), f64_bits((double)nsum), 0ull});
  };
  const unsigned long long* all = nullptr;
  size_t xs = 0;
  PeerXfer px;
  cudaError_t fe = cudaSuccess;
  if (peer_fits(stride)) {
    // over peer memory the channel fold puts, waits and folds itself
    if (exchange(rec, hdr(valid), &all, &xs, &px, W) != XCH_PEER) { *rc = DCT_ERR_DIST; return false; }
    bool fused = false;
    if (valid) {
      double* ps = (double*)rt_ws();
      cudaError_t e = launch_bn_plane_sums(x, dy, N, C, S, ps, st);
      if (e == cudaSuccess) e = launch_bn_fold_xchg(ps, N, C, px, D.fold, st);
      fused = e == cudaSuccess;
      if (!fused) { cudaGetLastError(); px.h = hdr(false); }
    }
    if (!fused)                                     // still puts and waits: an invalid header
      fe = launch_pdl(k_peer_fold_sums, dim3(fold_blocks((uint64_t)nsum + 1)), dim3(256), 0, st, px, nsum, D.fold);
  } else {
    if (valid) {
      double* ps = (double*)rt_ws();
      cudaError_t e = launch_bn_plane_sums(x, dy, N, C, S, ps, st);
      if (e == cudaSuccess) e = launch_bn_fold(ps, N, C, rec, st);     // [C][2] sums straight into the record
      if (!rt_cuda_ok(e, W)) valid = false;
    }
    const Xch how = exchange(rec, hdr(valid), &all, &xs, &px, W);
    if (how == XCH_FAIL) { *rc = DCT_ERR_DIST; return false; }
    fe = launch_pdl(k_fold_sums, dim3((nsum + 1 + 255) / 256), dim3(256), 0, st, (const double*)all, (uint64_t)xs,
                    D.world, nsum, D.fold, device_error_word());
  }
  if (!rt_cuda_ok(fe, W)) {
    *rc = DCT_ERR_CUDA;
    return false;
  }
  return true;
}
}  // namespace

// BatchNorm training forward over this rank's N samples: statistics over all
// ranks' samples (global count), running stats updated identically on every rank
DCT_API int dct_dist_batchnorm_forward_train(void* x, void* gamma, void* beta, void* running_mean,
                                             void* running_var, void* batch_mean, void* batch_var, void* y,
                                             uint32_t N, uint32_t C, uint32_t S, float eps, float momentum) {
  DLOCK;
  const char* W = "dct_dist_batchnorm_forward_train";
  if (!need_comm(W)) return DCT_ERR_DIST;
  if (C == 0) { note_error(DCT_ERR_ARG, "dct_dist_batchnorm_forward_train: C == 0"); return DCT_ERR_ARG; }
  Buffer *bx = live(x), *bg = live(gamma), *bb = live(beta), *rm = live(running_mean), *rv = live(running_var),
         *bm = live(batch_mean), *bvv = live(batch_var), *by = live(y);
  const uint64_t n = (uint64_t)N * C * S;
  const bool valid = bx && bg && bb && rm && rv && bm && bvv && by && bx->count >= n && by->count >= n &&
                     bg->count >= C && bb->count >= C && rm->count >= C && rv->count >= C && bm->count >= C &&
                     bvv->count >= C;
  int rc = 0;
  if (!bn_exchange(valid ? bx->d : nullptr, nullptr, N, C, S, valid, W, &rc)) return rc;
  if (!valid) { note_error(DCT_ERR_ARG, "dct_dist_batchnorm_forward_train: invalid handles or sizes on this rank"); return DCT_ERR_ARG; }
  cudaStream_t st = rt_stream();
  cudaError_t e = launch_bn_stats_final(D.fold, C, 0.0, bm->d, bvv->d, rm->d, rv->d, true, momentum, st, D.fold + 2 * C);
  if (e == cudaSuccess) e = launch_bn_forward(bx->d, bm->d, bvv->d, bg->d, bb->d, by->d, N, C, S, eps, n, st);
  return rt_cuda_ok(e, W) ? 0 : DCT_ERR_CUDA;
}

// BatchNorm backward over this rank's N samples: dgamma / dbeta summed over
// all ranks (identical everywhere), dx of the local samples with m = global N*S
DCT_API int dct_dist_batchnorm_backward(void* x, void* dy, void* batch_mean, void* batch_var, void* gamma,
                                        void* dgamma, void* dbeta, void* dx, uint32_t N, uint32_t C, uint32_t S,
                                        float eps) {
  DLOCK;
  const char* W = "dct_dist_batchnorm_backward";
  if (!need_comm(W)) return DCT_ERR_DIST;
  if (C == 0) { note_error(DCT_ERR_ARG, "dct_dist_batchnorm_backward: C == 0"); return DCT_ERR_ARG; }
  Buffer *bx = live(x), *bd = live(dy), *bm = live(batch_mean), *bv = live(batch_var), *bg = live(gamma),
         *dg = live(dgamma), *db = live(dbeta), *bo = live(dx);
  const uint64_t n = (uint64_t)N * C * S;
  const bool valid = bx && bd && bm && bv && bg && dg && db && bo && bx->count >= n && bd->count >= n &&
                     bo->count >= n && bm->count >= C && bv->count >= C && bg->count >= C && dg->count >= C &&
                     db->count >= C;
  int rc = 0;
  if (!bn_exchange(valid ? bx->d : nullptr, valid ? bd->d : nullptr, N, C, S, valid, W, &rc)) return rc;
  if (!valid) { note_error(DCT_ERR_ARG, "dct_dist_batchnorm_backward: invalid handles or sizes on this rank"); return DCT_ERR_ARG; }
  cudaStream_t st = rt_stream();
  cudaError_t e = launch_bn_bwd_final(D.fold, C, bm->d, bv->d, eps, dg->d, db->d, st);
  if (e == cudaSuccess)
    e = launch_bn_backward_dx(bx->d, bd->d, bm->d, bv->d, bg->d, dg->d, db->d, bo->d, N, C, S, eps, n, st,
                              D.fold + 2 * C);
  return rt_cuda_ok(e, W) ? 0 : DCT_ERR_CUDA;
}

}  // extern "C"
