/*
 * dct_cuda.h -- C-ABI of libdct_cuda.so, the B200 (sm_100a) drop-in for the
 * native engine of raviadi12/directcompute_torch.
 *
 * The reference Python (`nn_engine.py`) loads its engine with
 * `ctypes.CDLL(_find_resource("engine.dll"))` (nn_engine.py:42) and binds the
 * symbols below with the argtypes of nn_engine.py:43-119 and :133-134.  Each
 * declaration names the reference definition it replaces (engine.cpp:line).
 * Argument meaning, ownership and the quiet-failure error behaviour are the
 * reference's; what each call does on the device is described beside it.
 *
 * Symbols prefixed `dct_` are extensions with no counterpart in engine.cpp:
 * error reporting, device timing, raw-pointer interop, the NumPy-semantics ops
 * (broadcast binary ops, exp/log/tanh, axis and full reductions, fused
 * softmax+cross-entropy, fused Adam, fused BatchNorm) and multi-GPU sharding.
 *
 * Buffers are opaque handles to fp32 device arrays (labels and counters are
 * stored as 32-bit words in the same buffers, as the reference does).  All
 * work is enqueued in order on one CUDA stream per process; ReadBuffer,
 * SGDBatchClipped, SyncGPU, dct_synchronize and dct_timer_stop_ms wait for it.
 */
#ifndef DCT_CUDA_H
#define DCT_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#include <wchar.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DCT_API __attribute__((visibility("default")))
#define DCT_ABI_VERSION 1

/* error codes returned by dct_* calls and by dct_error_code() */
enum {
  DCT_OK = 0,
  DCT_ERR_NO_DEVICE = 1,      /* no CUDA device / InitEngine failed */
  DCT_ERR_HANDLE = 2,         /* a handle is not a live buffer */
  DCT_ERR_SIZE = 3,           /* a buffer is smaller than the dispatch touches */
  DCT_ERR_ARG = 4,            /* bad shape / count / view list */
  DCT_ERR_CUDA = 5,           /* a CUDA call or launch failed (message has the reason) */
  DCT_ERR_UNKNOWN_SHADER = 6, /* RunShader of a name without a compiled kernel */
  DCT_ERR_UNSUPPORTED = 7,    /* entry point outside this library's scope */
  DCT_ERR_DIST = 8,           /* NCCL / sharding error or timeout */
};

/* engine.cpp:14-21 GPUInfo, read by nn_engine.py:124-140 */
typedef struct DctGPUInfo {
  uint32_t vendorId;       /* 0x10DE */
  uint32_t deviceId;
  uint64_t dedicatedVRAM;  /* cudaDeviceProp::totalGlobalMem */
  uint64_t sharedMemory;
  uint32_t isIntegrated;   /* 0: nn_engine.py selects its dGPU code paths */
  char description[128];   /* device name */
} DctGPUInfo;

/* engine.cpp:940-950 SeqCmd, mirrored by nn_engine.py:2490-2502 (200 bytes on x86-64) */
typedef struct DctSeqCmd {
  void* shader;            /* pointer returned by ResolveShader */
  void* srvs[8];
  uint32_t srvCount;
  void* uavs[4];
  uint32_t uavCount;
  uint32_t threads[3];
  uint8_t cbData[64];
  uint32_t cbSize;
  uint32_t pad[1];
} DctSeqCmd;

/* ---- device ------------------------------------------------------------- */
/* engine.cpp:61-129. Picks $DCT_DEVICE, else $LOCAL_RANK, else the current CUDA
 * device; creates the stream. false when no device is visible. */
DCT_API bool InitEngine(void);
/* engine.cpp:132-134 */
DCT_API void GetGPUInfo(DctGPUInfo* out);
/* engine.cpp:136-152. Marks the built-in CUDA kernel `name` usable by RunShader;
 * the HLSL file at `path` is not read. false for names with no kernel here. */
DCT_API bool CompileShader(const char* name, const wchar_t* path);
/* engine.cpp:154-170. Arbitrary HLSL cannot run on CUDA: always false. */
DCT_API bool CompileShaderEx(const char* name, const wchar_t* path, const char* entryPoint);
/* engine.cpp:325-327: submits queued work, never waits */
DCT_API void FlushGPU(void);
/* engine.cpp:331-347: waits for all queued work */
DCT_API void SyncGPU(void);

/* ---- buffers ------------------------------------------------------------- */
/* engine.cpp:201-253. count fp32 elements (refcount 1), from the size-keyed
 * pool when possible; `data` (nullable) is uploaded. null on count 0 / OOM. */
DCT_API void* CreateBuffer(float* data, uint32_t count);
/* engine.cpp:255-258 */
DCT_API void AddRefBuffer(void* handle);
/* engine.cpp:261-265: uploads `count` floats; `data` may be reused on return */
DCT_API void UpdateBuffer(void* handle, float* data);
/* engine.cpp:284-290: refcount--, at zero the buffer returns to the pool
 * (per-size caps of engine.cpp:186-197) or is freed */
DCT_API void ReleaseBuffer(void* handle);
/* engine.cpp:676-685 */
DCT_API void ReleaseBufferBatch(void** handles, uint32_t count);
/* engine.cpp:292-321: blocking copy of all `count` floats to `dst` */
DCT_API void ReadBuffer(void* handle, float* dst);
/* engine.cpp:349-354: zero bits */
DCT_API void ClearBuffer(void* handle);

/* ---- kernels by name ------------------------------------------------------- */
/* engine.cpp:396-401. `threads` are the reference's group counts; the CUDA
 * kernels derive their own grid from the cbuffer fields and the groups'
 * index space (groups x [numthreads]). Unknown names return silently and set
 * DCT_ERR_UNKNOWN_SHADER. Names: add_bias bias_relu relu relu_grad relu6
 * relu6_grad leaky_relu leaky_relu_grad sigmoid sigmoid_grad add scale_add
 * grad_accum bias_grad global_avg_pool global_avg_pool_backward softmax loss
 * softmax_ce_grad argmax_correct accumulate_scalar rms grad_sq_reduce
 * grad_norm_final sgd sgd_clipped adam batchnorm_mean_var batchnorm_forward
 * batchnorm_backward_reduce batchnorm_backward_dx dice_loss dice_loss_sums
 * dice_loss_grad upsample upsample_backward concat_insert slice
 * maxpool_forward maxpool_backward conv_reshape conv_grad_reshape
 * conv_grad_reshape_relu, plus the extension names dct_unary dct_binary
 * dct_reduce dct_reduce_all dct_softmax_ce (cbuffer layouts in runtime.cu).
 * A buffer smaller than the largest index a dispatch touches is refused
 * (DCT_ERR_SIZE) rather than overrun; maxpool_backward drops indices past its
 * UAV, as D3D11 drops out-of-range UAV writes. */
DCT_API void RunShader(const char* name, void** srvs, uint32_t srvCount, void** uavs, uint32_t uavCount,
                       uint32_t* threads, void* cb, uint32_t cbSize);
/* engine.cpp:404-406 (alias) */
DCT_API void RunShaderRaw(const char* name, void** srvs, uint32_t srvCount, void** uavs, uint32_t uavCount,
                          uint32_t* threads, void* cb, uint32_t cbSize);
/* engine.cpp:409-416 */
DCT_API void* RunShaderAlloc(const char* name, void** srvs, uint32_t srvCount, uint32_t outCount,
                             uint32_t* threads, void* cb, uint32_t cbSize);
/* engine.cpp:419-426 */
DCT_API void* RunShaderAlloc2(const char* name, void** srvs, uint32_t srvCount, uint32_t outCount,
                              void* extraUav, uint32_t* threads, void* cb, uint32_t cbSize);

/* ---- optimizers ------------------------------------------------------------- */
/* engine.cpp:436-485: w -= lr * clamp(g, +-clip) for every (param, grad) pair,
 * one multi-tensor launch */
DCT_API void SGDBatch(void** params, void** grads, uint32_t* sizes, uint32_t numParams, float lr, float clip);
/* engine.cpp:494-614: global grad norm (float64), clip scale
 * max/(norm+1e-6) when norm > max, w -= lr*g*scale; returns the norm (blocks) */
DCT_API float SGDBatchClipped(void** params, void** grads, uint32_t* sizes, uint32_t numParams, float lr,
                              float maxNorm);

/* ---- outside the hot path: exported so nn_engine.py binds; null + DCT_ERR_UNSUPPORTED */
DCT_API void* MatMulAlloc(void* a, void* b, uint32_t M, uint32_t K, uint32_t N, uint32_t flags); /* engine.cpp:741-747 */
DCT_API void* ConvForwardFused(void* x, void* f, void* bias, uint32_t batch, uint32_t inC, uint32_t inH,
                               uint32_t inW, uint32_t outC, uint32_t kH, uint32_t kW, uint32_t stride,
                               uint32_t padding, uint32_t actType, void** pIm2col); /* engine.cpp:751-799 */
DCT_API void ConvBackwardFused(void* go, void* fo, void* x, void* f, void* im2col, uint32_t batch, uint32_t inC,
                               uint32_t inH, uint32_t inW, uint32_t outC, uint32_t kH, uint32_t kW,
                               uint32_t stride, uint32_t padding, uint32_t actType, uint32_t xg, uint32_t fg,
                               uint32_t bg, void** pDF, void** pDB, void** pDI); /* engine.cpp:802-876 */

/* ---- max pooling ---------------------------------------------------------------- */
/* engine.cpp:880-902: output and index buffers of batch*inC*outH*outW with
 * outH = (inH - pool)/stride + 1 (likewise outW); per output the window's first
 * maximum above -1e30 (strict >, NaN never selected) and its flat input index,
 * 0xFFFFFFFF when nothing beat -1e30; *pIdx = the index buffer (released if
 * pIdx is null).  Returns null (DCT_ERR_ARG) for pool or stride 0 or a pool
 * larger than the input. */
DCT_API void* MaxPoolForwardFused(void* x, uint32_t batch, uint32_t inC, uint32_t inH, uint32_t inW,
                                  uint32_t pool, uint32_t stride, void** pIdx);
/* engine.cpp:905-929: dInput of xSize floats = 0 except dInput[idx[o]] =
 * go[o] (indices past xSize dropped), then releases idx.  Index buffers from
 * MaxPoolForwardFused with non-overlapping windows take a one-pass gather;
 * the result is the same for any index contents. */
DCT_API void* MaxPoolBackwardFused(void* go, void* idx, uint32_t batch, uint32_t inC, uint32_t outH,
                                   uint32_t outW, uint32_t xSize);

/* ---- pool -------------------------------------------------------------------- */
DCT_API void WarmPool(uint32_t* sizes, uint32_t numSizes, uint32_t copies); /* engine.cpp:617-635 */
DCT_API void GetPoolStats(uint64_t* hits, uint64_t* misses);                /* engine.cpp:637-640 */
DCT_API void ResetPoolStats(void);                                          /* engine.cpp:642-645 */
DCT_API uint64_t GetPoolMemory(void);                                       /* engine.cpp:648-650 */
DCT_API void DrainPool(void);                                               /* engine.cpp:654-673 */

/* ---- graph replay ---------------------------------------------------------------- */
/* engine.cpp:934-937: a stable kernel-descriptor pointer for SeqCmd.shader */
DCT_API void* ResolveShader(const char* name);
/* engine.cpp:952-966 */
DCT_API void RunSequence(DctSeqCmd* cmds, uint32_t count);
/* engine.cpp:969-977 */
DCT_API void RunSequenceWithSGD(DctSeqCmd* cmds, uint32_t cmdCount, void** params, void** grads,
                                uint32_t* sizes, uint32_t numParams, float lr, float clip);

/* ======================= extensions (no engine.cpp counterpart) ================= */
DCT_API const char* dct_last_error(void);   /* message of the last failure ("" if none) */
DCT_API int dct_error_code(void);           /* DCT_ERR_* of the last failure, 0 if none */
DCT_API void dct_clear_error(void);
DCT_API int dct_version(void);              /* DCT_ABI_VERSION */
DCT_API int dct_device(void);               /* CUDA ordinal in use, -1 if none */
DCT_API int dct_sm_count(void);
DCT_API void* dct_stream(void);             /* the library's cudaStream_t */
DCT_API int dct_pci_bus_id(char* out, int len);   /* "0000:xx:00.0" of the device in use */
DCT_API int dct_synchronize(void);
/* CUDA events on the library's stream: start, then stop returns elapsed ms (waits) */
DCT_API int dct_timer_start(void);
DCT_API float dct_timer_stop_ms(void);

/* buffers beyond 2^32 elements, raw pointers, partial copies, pinned host memory */
DCT_API void* dct_create_buffer(uint64_t count);
DCT_API void* dct_buffer_device_ptr(void* handle);
DCT_API uint64_t dct_buffer_count(void* handle);
DCT_API int dct_buffer_refcount(void* handle);
/* non-owning handle over caller device memory (released with ReleaseBuffer, never freed) */
DCT_API void* dct_wrap_device_ptr(void* dptr, uint64_t count);
DCT_API int dct_copy_h2d(void* handle, const void* src, uint64_t offset, uint64_t count);   /* async */
DCT_API int dct_copy_d2h(void* handle, void* dst, uint64_t offset, uint64_t count);         /* waits */
DCT_API void* dct_host_alloc(uint64_t bytes);   /* pinned */
DCT_API void dct_host_free(void* p);

/* synthetic data: Philox4x32-10 fill of the whole buffer; dist 0 = uniform [a,b),
 * 1 = normal(mean a, std b); element i uses counter (i/4, offset), key seed */
DCT_API int dct_fill_random(void* handle, uint64_t seed, uint64_t offset, int dist, float a, float b);
/* x[idx[i]] = vals[i] (host arrays), e.g. outlier injection */
DCT_API int dct_scatter(void* handle, const int64_t* idx, const float* vals, uint64_t k);

/* unary ops: 0 relu 1 relu6 2 leaky_relu(alpha) 3 sigmoid 4 exp 5 log(|x|+1) 6 tanh 7 neg 8 abs */
DCT_API int dct_unary(int op, void* x, void* y, uint64_t n, float alpha);
/* NumPy-broadcast binary op: 20 add 21 sub 22 mul 23 div 24 maximum 25 minimum;
 * gradient masks 27 pick_max / 28 pick_min = 1.0 where maximum / minimum(a, b)
 * routes the gradient to a (a >= b resp. a <= b, or a is NaN), else 0.0.
 * Same shapes only: 19 sigmoid_grad(dy, y) = dy*y*(1-y), 29 exp_grad(g, y) = g*y,
 * 30 tanh_grad(g, y) = g*(1-y*y), 31 log_abs1p_grad(g, x) = g*sign(x)/(|x|+1),
 * 32 copy (out = a broadcast to the output shape; b is not used but must be valid).
 * Shapes are right-aligned; out has the broadcast shape (<= 8 dims). */
DCT_API int dct_binary(int op, void* a, const int64_t* a_shape, int a_ndim, void* b, const int64_t* b_shape,
                       int b_ndim, void* out);
/* broadcast gradient: out (t_shape) = g (g_shape) summed over the dims where
 * t_shape (right-aligned, padded with 1s) has extent 1 and g does not; float64
 * accumulation rounded once (the reverse of NumPy broadcasting) */
DCT_API int dct_sum_to_shape(void* g, const int64_t* g_shape, int g_ndim, const int64_t* t_shape, int t_ndim,
                             void* out);
/* backward of bias + ReLU over [rows, cols] in one pass (replaces the relu_grad
 * then bias_grad dispatches of BiasReLUFunc.backward, nn_engine.py:1091-1106;
 * nn_relu_grad.hlsl:6-9, nn_bias_grad.hlsl:8-29): dx = out > 0 ? grad : 0 and
 * db[c] = sum over rows of dx[r, c] (float64, rounded once).  Results equal the
 * two dispatches bit for bit.  dx may be grad itself.  RunSequence fuses a
 * relu_grad command followed by a bias_grad over its output the same way. */
DCT_API int dct_bias_relu_backward(void* grad, void* out, void* dx, void* db, uint32_t rows, uint32_t cols);
/* out (out_shape) = x (x_shape) broadcast NumPy-style (the reverse of dct_sum_to_shape) */
DCT_API int dct_broadcast_to(void* x, const int64_t* x_shape, int x_ndim, const int64_t* out_shape, int out_ndim,
                             void* out);
/* reduce x viewed as [outer, len, inner] over len: 0 sum 1 mean 2 max 3 argmax 4 min
 * 5 argmin 6 sum of squares; float64 accumulation; arg ops write int32 to out_idx
 * (or to out when out_idx is null); max/min also write indices when out_idx is set.
 * Empty operands follow NumPy: with len 0, sum writes 0 and mean NaN, and the
 * extremes and arg ops return DCT_ERR_ARG and write nothing; with outer or inner 0
 * there is nothing to write. */
DCT_API int dct_reduce(int op, void* x, uint64_t outer, uint64_t len, uint64_t inner, void* out, void* out_idx);
/* full reduction of n elements (sum, mean, max, min, sumsq) into out[0]; the
 * float64 value is returned in *host_out64 when non-null (waits).  n = 0 gives 0
 * for the sums and NaN for the mean; max and min return DCT_ERR_ARG. */
DCT_API int dct_reduce_all(int op, void* x, uint64_t n, void* out, double* host_out64);
/* fused row softmax + cross-entropy forward and backward in one pass:
 * probs, dlogits = (p - onehot)/grad_div, loss[0] = sum(ce)/loss_div, logprobs;
 * any output may be null; labels are float (reference layout) or int32.  A
 * divisor of 0 means `rows`; with rows = 0 the loss is 0 / loss_div (NaN for an
 * empty batch, as nn_loss.hlsl:41 computes it). */
DCT_API int dct_softmax_ce(void* logits, void* labels, int labels_int32, uint32_t rows, uint32_t K, void* probs,
                           void* dlogits, void* loss, void* logprobs, float loss_div, float grad_div);
/* nn_adam.hlsl semantics; step_size carries lr and the bias correction */
DCT_API int dct_adam(void* w, void* m, void* v, void* grad, uint64_t n, float step_size, float beta1, float beta2,
                     float eps, float weight_decay, float clip);
DCT_API int dct_adam_batch(void** w, void** m, void** v, void** grads, const uint32_t* sizes, uint32_t n,
                           float step_size, float beta1, float beta2, float eps, float weight_decay, float clip);
/* BatchNorm training forward (stats + running-stat update + normalize) and
 * backward (dgamma, dbeta, dx) over NCHW with S = H*W */
DCT_API int dct_batchnorm_forward_train(void* x, void* gamma, void* beta, void* running_mean, void* running_var,
                                        void* batch_mean, void* batch_var, void* y, uint32_t N, uint32_t C,
                                        uint32_t S, float eps, float momentum);
DCT_API int dct_batchnorm_backward(void* x, void* dy, void* batch_mean, void* batch_var, void* gamma,
                                   void* dgamma, void* dbeta, void* dx, uint32_t N, uint32_t C, uint32_t S,
                                   float eps);

/* BatchNorm training forward that allocates nothing.  No counterpart in the
 * reference: it is for callers that cannot let this library allocate device
 * memory (a process whose HBM is already owned by its own allocator or arena,
 * or one held to a fixed memory budget).  Same math and kernels as
 * dct_batchnorm_forward_train, but every buffer is a caller-owned device
 * pointer, work goes on `stream` (null = the legacy default stream), and the
 * float64 partial sums live in a fixed file-scope device array of 2 MiB +
 * 64 KiB that every GPU loading the library keeps until exit.  Limit:
 * N*C <= 131072 and C <= 4096, otherwise DCT_ERR_SIZE with a message and
 * nothing is launched.  The first call on a device looks up the array's device
 * address; make it before any stream capture.  All calls share the array:
 * calls that overlap on the GPU race and must be serialised. */
DCT_API int dct_batchnorm_forward_train_noalloc(const float* x, const float* gamma, const float* beta,
                                                float* running_mean, float* running_var, float* batch_mean,
                                                float* batch_var, float* y, uint32_t N, uint32_t C, uint32_t S,
                                                float eps, float momentum, void* stream);

/* ======================= sharding over NCCL (one process per GPU) ==============
 * No counterpart in the reference, which drives one D3D11 device
 * (engine.cpp:61-129).  Each rank holds one contiguous shard of the sharded
 * axis; ops whose result depends on other shards make one NCCL all-gather of
 * small fixed-size records, folded on the device in rank order (identical
 * results on every rank; at world size 1 bit-identical to the single-GPU
 * entry points).  Every rank must make the same dct_dist_* calls in the same
 * order with the same outer/inner/C/S/op.  A rank whose own arguments are bad
 * still takes part in the exchange and returns DCT_ERR_ARG; the other ranks
 * get DCT_ERR_DIST at their next wait.  While a communicator is active every
 * wait of the library is bounded by the init timeout and aborts the
 * communicator when it expires or NCCL reports an asynchronous error.
 * Other ops (elementwise, axis -1 reductions, Adam) shard with no exchange. */
DCT_API int dct_dist_available(void);          /* 1 if an NCCL library can be loaded */
DCT_API int dct_dist_nccl_version(void);       /* NCCL_VERSION_CODE of that library, 0 if none */
/* balanced contiguous split: shard `rank` of n items is [*offset, *offset + *count) */
DCT_API int dct_dist_shard(uint64_t n, int world, int rank, uint64_t* offset, uint64_t* count);
DCT_API int dct_dist_unique_id(void* out, int len);   /* rank 0: 128-byte id to send to every rank */
DCT_API int dct_dist_init(const void* id, int len, int nranks, int rank, double timeout_s);
DCT_API int dct_dist_finalize(void);
DCT_API int dct_dist_rank(void);    /* -1 without a communicator */
DCT_API int dct_dist_world(void);   /* 0 without a communicator */
/* 1 when the sharded ops exchange records through mapped peer memory (NVLink,
 * CUDA IPC), 0 when they use NCCL all-gathers (or without a communicator) */
DCT_API int dct_dist_peer_active(void);
/* in-place fp32 all-reduce of buf[0:count]: op 0 sum, 1 mean, 2 max, 4 min */
DCT_API int dct_dist_allreduce(void* buf, uint64_t count, int op);
DCT_API int dct_dist_broadcast(void* buf, uint64_t count, int root);
DCT_API int dct_dist_barrier(void);
/* dct_reduce over a sharded middle axis: x is [outer, len, inner], this rank's
 * slice [len_offset, len_offset + len) of an axis of extent len_total (the
 * ranks' slices tile it in rank order; checked on the device).  out / out_idx
 * as dct_reduce, identical on every rank; indices are global (< 2^31). */
DCT_API int dct_dist_reduce(int op, void* x, uint64_t outer, uint64_t len, uint64_t inner, uint64_t len_offset,
                            uint64_t len_total, void* out, void* out_idx);
/* dct_reduce_all over every rank's n elements (0 sum, 1 mean, 2 max, 4 min, 6 sumsq) */
DCT_API int dct_dist_reduce_all(int op, void* x, uint64_t n, void* out, double* host_out64);
/* dct_softmax_ce over this rank's rows; pass the global batch as grad_div and
 * loss_div: loss[0] = (sum of every rank's row losses) / loss_div */
DCT_API int dct_dist_softmax_ce(void* logits, void* labels, int labels_int32, uint32_t rows, uint32_t K,
                                void* probs, void* dlogits, void* loss, void* logprobs, float loss_div,
                                float grad_div);
/* BatchNorm over this rank's N samples with statistics of all ranks' samples */
DCT_API int dct_dist_batchnorm_forward_train(void* x, void* gamma, void* beta, void* running_mean,
                                             void* running_var, void* batch_mean, void* batch_var, void* y,
                                             uint32_t N, uint32_t C, uint32_t S, float eps, float momentum);
DCT_API int dct_dist_batchnorm_backward(void* x, void* dy, void* batch_mean, void* batch_var, void* gamma,
                                        void* dgamma, void* dbeta, void* dx, uint32_t N, uint32_t C, uint32_t S,
                                        float eps);

/* self-test of the device-side bounded wait: one block waits on a barrier
 * phase that nothing completes, gives up after `spins` polls, sets the device
 * error word and exits; the next wait returns DCT_ERR_CUDA and the context
 * stays usable */
DCT_API int dct_selftest_bounded_wait(uint32_t spins);

#ifdef __cplusplus
}
#endif
#endif /* DCT_CUDA_H */
