"""NumPy restatement of the reference's hot-path HLSL shaders (test oracle only).

Every function follows one `nn_*.hlsl` compute shader of raviadi12/directcompute_torch;
the docstring cites the file:line.  Buffers are flat NumPy arrays (float32, or a
uint32 view where the shader declares `uint`), the cbuffer arrives as the same
little-endian 32-bit words `nn_engine._dispatch` packs (`nn_engine.py:458-470`),
and `groups` is the (x, y, z) group count the Python side dispatches.

Arithmetic rules the CUDA library is held to:

* Elementwise shaders: fp32, each `*`, `+`, `/` rounded separately (no fused
  multiply-add), IEEE division and square root.  Results are BIT-EXACT targets.
* `max(0, x)` / `min(max(x, 0), 6)` are restated as explicit selects
  (`x > 0 ? x : +0`), which is what HLSL's IEEE maxNum gives for NaN (-> 0).
* Reductions: the shaders accumulate in fp32 in a driver-chosen order; the
  oracle accumulates in float64 and rounds once where the shader stores, and the
  CUDA library is held to rel 1e-5 of that.  Post-reduction scalar math
  (means, variances, norms, clip scales, running statistics) is done in float64
  and rounded once at the store.
* Transcendentals (`exp`, `log`): the oracle evaluates in float64 and rounds,
  the CUDA library is held to <= 2 ulp (per element) of that.
"""
from __future__ import annotations

import struct

import numpy as np

F32 = np.float32
F64 = np.float64


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def u2f(u: int) -> np.float32:
    """`asfloat(uint)`: reinterpret 32 bits as an IEEE float (nn_engine.py:10-11 inverse)."""
    return np.frombuffer(struct.pack("<I", int(u) & 0xFFFFFFFF), dtype=np.float32)[0]


def f2u(f: float) -> int:
    """`float_to_uint` of nn_engine.py:10-11 (Python float rounded to the nearest f32)."""
    return struct.unpack("<I", struct.pack("<f", float(f)))[0]


def _hlsl_f2u(x: np.ndarray) -> np.ndarray:
    """HLSL `(uint)float`: truncation toward zero, NaN and negatives -> 0, saturating."""
    x = np.asarray(x, dtype=np.float64)
    out = np.where(np.isnan(x) | (x <= 0), 0.0, np.minimum(np.floor(x), 4294967295.0))
    return out.astype(np.uint64)


def _relu(x: np.ndarray) -> np.ndarray:
    return np.where(x > 0, x, F32(0.0)).astype(F32)


def _lim(count: int, groups, tpg: int = 256) -> int:
    """Threads that pass `id.x < count` when `groups[0]` groups of `tpg` threads run."""
    return int(max(0, min(int(count), int(groups[0]) * tpg)))


# ---------------------------------------------------------------------------
# elementwise shaders
# ---------------------------------------------------------------------------

def add_bias(A, B, M, N, limit=None):
    """nn_add_bias.hlsl:6-10 -- C[i] = A[i] + B[i % N] for i < M*N."""
    n = M * N if limit is None else min(M * N, limit)
    i = np.arange(n, dtype=np.int64)
    return (A[:n] + B[i % N]).astype(F32)


def bias_relu(A, B, M, N, limit=None):
    """nn_bias_relu.hlsl:8-12 -- C[i] = max(0, A[i] + B[i % N])."""
    return _relu(add_bias(A, B, M, N, limit))


def relu(A, n_out):
    """nn_relu.hlsl:4-6 -- B[i] = max(0, A[i]); no cbuffer, no bounds check.

    D3D11 discards writes past the UAV and reads past the SRV return 0, so the
    written range is the output buffer (clamped to the dispatch) and inputs past
    A's end read as 0.
    """
    out = np.zeros(n_out, dtype=F32)
    k = min(n_out, A.size)
    out[:k] = _relu(A[:k])
    return out


def relu_grad(grad_out, inp, count):
    """nn_relu_grad.hlsl:6-9 -- grad_in[i] = input[i] > 0 ? grad_out[i] : 0."""
    return np.where(inp[:count] > 0, grad_out[:count], F32(0.0)).astype(F32)


def relu6(x, count):
    """nn_relu6.hlsl:6-10 -- min(max(x, 0), 6) (NaN -> 0 under IEEE maxNum)."""
    x = x[:count]
    return np.where(x > 0, np.where(x < 6, x, F32(6.0)), F32(0.0)).astype(F32)


def relu6_grad(dy, x, count):
    """nn_relu6_grad.hlsl:7-11 -- (0 < x < 6) ? dy : 0."""
    x = x[:count]
    return np.where((x > 0) & (x < 6), dy[:count], F32(0.0)).astype(F32)


def leaky_relu(x, count, alpha):
    """nn_leaky_relu.hlsl:10-14 -- x > 0 ? x : x * alpha."""
    x = x[:count]
    return np.where(x > 0, x, x * F32(alpha)).astype(F32)


def leaky_relu_grad(dy, x, count, alpha):
    """nn_leaky_relu_grad.hlsl:11-16 -- dy * (x > 0 ? 1 : alpha)."""
    x = x[:count]
    return (dy[:count] * np.where(x > 0, F32(1.0), F32(alpha)).astype(F32)).astype(F32)


def sigmoid_f64(x, count):
    """nn_sigmoid.hlsl:9-12 -- 1 / (1 + exp(-x)), evaluated in float64 and rounded."""
    x = x[:count].astype(F64)
    with np.errstate(over="ignore"):
        return (1.0 / (1.0 + np.exp(-x))).astype(F32)


def sigmoid_grad(dy, y, count):
    """nn_sigmoid_grad.hlsl:10-14 -- dy * y * (1 - y), left to right in fp32."""
    y = y[:count]
    return ((dy[:count] * y) * (F32(1.0) - y)).astype(F32)


def add(A, B, M, N):
    """nn_add.hlsl:6-7 -- C[i] = A[i] + B[i] for i < M*N."""
    n = M * N
    return (A[:n] + B[:n]).astype(F32)


def scale_add(A, B, count, alpha, beta):
    """nn_scale_add.hlsl:7-10 -- alpha*A + beta*B (two products, one add, unfused)."""
    return (F32(alpha) * A[:count] + F32(beta) * B[:count]).astype(F32)


def grad_accum(accum, grad, count):
    """nn_grad_accum.hlsl:5-8 -- accum[i] = accum[i] + grad[i] (in place)."""
    return (accum[:count] + grad[:count]).astype(F32)


def global_avg_pool_backward(g, batch, C, S):
    """nn_global_avg_pool_backward.hlsl:14-19 -- dx[i] = g[i / S] / (float)S."""
    n = batch * C * S
    i = np.arange(n, dtype=np.int64)
    return (g[i // S] / F32(S)).astype(F32)


def softmax_ce_grad(p, labels, B, K, limit_x=None, limit_y=None):
    """nn_softmax_ce_grad.hlsl:6-11 -- (p - (label == col)) / (float)B over a 16x16 grid."""
    kx = K if limit_x is None else min(K, limit_x)
    by = B if limit_y is None else min(B, limit_y)
    P = p[: B * K].reshape(B, K)[:by, :kx]
    onehot = (labels[:by, None] == np.arange(kx, dtype=F32)[None, :]).astype(F32)
    return ((P - onehot) / F32(B)).astype(F32)


def accumulate_scalar(dst, src):
    """nn_accumulate_scalar.hlsl:6-8 -- dst[0] = dst[0] + src[0]."""
    return F32(dst[0] + src[0])


def sgd(w, g, count, lr, clip):
    """nn_sgd.hlsl:5-11 -- clamp g to [-clip, clip] (NaN passes), w -= lr * g."""
    g = g[:count].copy()
    g = np.where(g > F32(clip), F32(clip), g)
    g = np.where(g < -F32(clip), -F32(clip), g).astype(F32)
    return (w[:count] - F32(lr) * g).astype(F32)


def sgd_clipped(w, g, count, lr, scale):
    """nn_sgd_clipped.hlsl:15-20 -- w -= lr * g * scale, (lr*g) first."""
    return (w[:count] - (F32(lr) * g[:count]) * F32(scale)).astype(F32)


def adam(w, m, v, g, count, step_size, beta1, beta2, eps, wd, clip):
    """nn_adam.hlsl:18-34 -- clipped-gradient Adam(W); returns (w, m, v).

    m_t = b1*m + (1-b1)*g ; v_t = b2*v + ((1-b2)*g)*g ;
    w   = (w - wd*w) - (step*m_t) / (sqrt(v_t) + eps), every op rounded to fp32.
    `step_size` already folds lr and the bias correction (nn_engine.py:2220).
    """
    b1, b2 = F32(beta1), F32(beta2)
    g = g[:count]
    g = np.where(g > F32(clip), F32(clip), g)
    g = np.where(g < -F32(clip), -F32(clip), g).astype(F32)
    cw = w[:count]
    m_t = (b1 * m[:count] + (F32(1.0) - b1) * g).astype(F32)
    v_t = (b2 * v[:count] + ((F32(1.0) - b2) * g) * g).astype(F32)
    w_t = ((cw - F32(wd) * cw) - (F32(step_size) * m_t) / (np.sqrt(v_t) + F32(eps))).astype(F32)
    return w_t, m_t, v_t


def adam_step_size(lr, beta1, beta2, t):
    """AdamW.step's bias-corrected step size (nn_engine.py:2220), f64 then f32 bits."""
    step = lr * (1 - beta2 ** t) ** 0.5 / (1 - beta1 ** t)
    return u2f(f2u(step))


def batchnorm_forward(x, mean, var, gamma, beta, N, C, S, eps):
    """nn_batchnorm_forward.hlsl:18-34 -- y = ((x - m) * (1/sqrt(v+eps))) * g + b."""
    n = N * C * S
    c = (np.arange(n, dtype=np.int64) // S) % C
    rstd = (F32(1.0) / np.sqrt(var[:C] + F32(eps))).astype(F32)
    xhat = ((x[:n] - mean[c]) * rstd[c]).astype(F32)
    return (xhat * gamma[c] + beta[c]).astype(F32)


def batchnorm_backward_dx(x, dy, mean, var, gamma, dgamma, dbeta, N, C, S, eps, count=None):
    """nn_batchnorm_backward_dx.hlsl:20-38 -- dx = (g*rstd) * (dy - (db + xhat*dg) / m).

    m is the batch's N*S; `count` overrides it when x holds only some samples of
    the batch (a chunked check, or one rank's shard)."""
    n = N * C * S
    c = (np.arange(n, dtype=np.int64) // S) % C
    rstd = (F32(1.0) / np.sqrt(var[:C] + F32(eps))).astype(F32)
    xhat = ((x[:n] - mean[c]) * rstd[c]).astype(F32)
    m = F32(N * S if count is None else count)
    inner = ((dbeta[c] + xhat * dgamma[c]) / m).astype(F32)
    return ((gamma[c] * rstd[c]) * (dy[:n] - inner)).astype(F32)


def dice_loss_grad(pred, target, sums, batch, size, divisor=None):
    """nn_dice_loss_grad.hlsl:17-34 -- -2 * ((t*denom) - inter) / (denom*denom) / batch.

    `divisor` (default: batch) is the shader's batch divisor, for checking a
    slice of samples of a larger batch."""
    n = batch * size
    b = np.arange(n, dtype=np.int64) // size
    inter = sums[b * 3 + 0]
    denom = (sums[b * 3 + 1] + sums[b * 3 + 2] + F32(1e-6)).astype(F32)
    t = target[:n]
    num = (F32(-2.0) * (t * denom - inter)).astype(F32)
    return ((num / (denom * denom)) / F32(batch if divisor is None else divisor)).astype(F32)


# ---------------------------------------------------------------------------
# reductions (float64 accumulation, rounded once at the store)
# ---------------------------------------------------------------------------

def bias_grad(g, batch, classes, stride_i, stride_id, limit=None):
    """nn_bias_grad.hlsl:8-29 -- out[c] = sum_i g[i*stride_i + c*stride_id]."""
    k = classes if limit is None else min(classes, limit)
    i = np.arange(batch, dtype=np.int64)[:, None]
    c = np.arange(k, dtype=np.int64)[None, :]
    idx = i * stride_i + c * stride_id
    return g.astype(F64)[idx].sum(axis=0).astype(F32)


def global_avg_pool(x, batch, C, S, limit=None):
    """nn_global_avg_pool.hlsl:16-35 -- out[nc] = sum_s x[nc*S + s] / S."""
    k = batch * C if limit is None else min(batch * C, limit)
    return (x[: k * S].astype(F64).reshape(k, S).sum(axis=1) / S).astype(F32)


def softmax_f64(x, B, K, limit=None):
    """nn_softmax.hlsl:5-13 -- stable row softmax, max initialised to -1e30."""
    b = B if limit is None else min(B, limit)
    X = x[: b * K].astype(F64).reshape(b, K)
    mx = np.maximum(X.max(axis=1, initial=-1e30), -1e30)[:, None]
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        e = np.exp(X - mx)
        return (e / e.sum(axis=1, keepdims=True)).astype(F32)


def ce_loss_f64(logits, labels, B, K):
    """nn_loss.hlsl:11-43 -- mean over rows of -(x[label] - max - log(sum exp(x - max)))."""
    X = logits[: B * K].astype(F64).reshape(B, K)
    mx = np.maximum(X.max(axis=1, initial=-1e30), -1e30)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        lse = np.log(np.exp(X - mx[:, None]).sum(axis=1))
    lab = _hlsl_f2u(labels[:B])
    flat = np.arange(B, dtype=np.int64) * K + lab.astype(np.int64)
    xl = np.where(flat < logits.size, logits.astype(F64)[np.minimum(flat, logits.size - 1)], 0.0)
    return F32((-(xl - mx - lse)).sum() / B)


def argmax_correct(logits, labels, B, K, limit=None):
    """nn_argmax_correct.hlsl:10-26 -- strict `>` scan from j=1, first index wins."""
    b = B if limit is None else min(B, limit)
    X = logits[: b * K].reshape(b, K)
    best = X[:, 0].copy()
    idx = np.zeros(b, dtype=np.int64)
    for j in range(1, K):
        upd = X[:, j] > best
        best = np.where(upd, X[:, j], best)
        idx = np.where(upd, j, idx)
    lab = _hlsl_f2u(labels[:b]).astype(np.int64)
    return int((idx == lab).sum())


def rms(a, count):
    """nn_rms.hlsl:7-24 -- sqrt(sum(a^2) / count)."""
    s = (a[:count].astype(F64) ** 2).sum()
    return F32(np.sqrt(s / count))


def grad_sq_reduce(g, count, ngroups):
    """nn_grad_sq_reduce.hlsl:16-30 -- one partial sum of g^2 per 256-element group."""
    out = np.zeros(ngroups, dtype=F64)
    gg = g[:count].astype(F64) ** 2
    k = min(ngroups, (count + 255) // 256)
    pad = np.zeros(k * 256, dtype=F64)
    pad[: min(count, k * 256)] = gg[: k * 256]
    out[:k] = pad.reshape(k, 256).sum(axis=1)
    return out.astype(F32)


def grad_norm_final(partials, total, max_norm):
    """nn_grad_norm_final.hlsl:16-35 -- [norm, norm > max ? max/(norm+1e-6) : 1]."""
    norm = np.sqrt(partials[:total].astype(F64).sum())
    norm32 = F32(norm)
    mn = F32(max_norm)
    scale = F32(F64(mn) / (F64(norm32) + F64(F32(1e-6)))) if norm32 > mn else F32(1.0)
    return norm32, scale


def batchnorm_mean_var(x, N, C, S):
    """nn_batchnorm_mean_var.hlsl:19-52 -- per-channel mean, biased var = max(0, E[x^2]-mean^2)."""
    X = x[: N * C * S].astype(F64).reshape(N, C, S)
    cnt = N * S
    s1 = X.sum(axis=(0, 2))
    s2 = (X * X).sum(axis=(0, 2))
    mean = s1 / cnt
    var = np.maximum(0.0, s2 / cnt - mean * mean)
    return mean, var


def batchnorm_running(rm, rv, mean64, var64, N, S, momentum):
    """nn_batchnorm_mean_var.hlsl:54-59 -- momentum update with the unbiased variance."""
    cnt = N * S
    mom = F64(F32(momentum))
    unbiased = var64 * (cnt / max(1.0, cnt - 1.0))
    rm2 = ((1.0 - mom) * rm.astype(F64) + mom * mean64).astype(F32)
    rv2 = ((1.0 - mom) * rv.astype(F64) + mom * unbiased).astype(F32)
    return rm2, rv2


def batchnorm_backward_reduce(x, dy, mean, var, N, C, S, eps):
    """nn_batchnorm_backward_reduce.hlsl:21-60 -- dgamma = sum dy*xhat, dbeta = sum dy.

    Restated exactly in float64: sum(dy * (x - m)) * rstd with m, rstd the fp32
    statistics the shader reads.
    """
    X = x[: N * C * S].astype(F64).reshape(N, C, S)
    D = dy[: N * C * S].astype(F64).reshape(N, C, S)
    rstd = (F32(1.0) / np.sqrt(var[:C] + F32(eps))).astype(F32).astype(F64)
    m = mean[:C].astype(F64)
    dg = (D * (X - m[None, :, None])).sum(axis=(0, 2)) * rstd
    db = D.sum(axis=(0, 2))
    return dg.astype(F32), db.astype(F32)


def dice_sums(pred, target, batch, size):
    """nn_dice_loss_sums.hlsl:19-55 -- per sample (sum p*t, sum p, sum t)."""
    P = pred[: batch * size].astype(F64).reshape(batch, size)
    T = target[: batch * size].astype(F64).reshape(batch, size)
    return np.stack([(P * T).sum(axis=1), P.sum(axis=1), T.sum(axis=1)], axis=1)


def dice_loss(pred, target, batch, size):
    """nn_dice_loss.hlsl:19-53 -- 1 - 2*inter / (sum p + sum t + 1e-6)."""
    s = dice_sums(pred, target, batch, size)
    return (1.0 - 2.0 * s[:, 0] / (s[:, 1] + s[:, 2] + F64(F32(1e-6)))).astype(F32)


# ---------------------------------------------------------------------------
# dispatcher over the reference's cbuffer layouts
# ---------------------------------------------------------------------------

# ---------------------------------------------------------------------------
# layout shaders beside the path: nearest upsample, channel concat / slice,
# max pooling, and the conv output / gradient reshapes
# ---------------------------------------------------------------------------
NO_INDEX = np.uint32(0xFFFFFFFF)


def upsample(x, batch, C, inH, inW, outH, outW, sH, sW, limit=None):
    """nn_upsample.hlsl:15-33: Out[b,c,h,w] = X[b,c,h//sH,w//sW] (nearest, integer scales)
    for flat output index < min(batch*C*outH*outW, limit)."""
    total = batch * C * outH * outW
    n = total if limit is None else min(total, limit)
    i = np.arange(n, dtype=np.int64)
    w = i % outW
    t = i // outW
    h = t % outH
    bc = t // outH
    src = (bc * inH + h // sH) * inW + w // sW
    return np.asarray(x, F32)[src]


def upsample_backward(dy, batch, C, inH, inW, outH, outW, sH, sW, limit=None):
    """nn_upsample_backward.hlsl:15-45: DX[b,c,h,w] = sum over the sH x sW block of DY
    (rows outer, columns inner, skipping positions past outH / outW), accumulated in
    fp32 from 0.0f in that order."""
    total = batch * C * inH * inW
    n = total if limit is None else min(total, limit)
    i = np.arange(n, dtype=np.int64)
    w = i % inW
    t = i // inW
    h = t % inH
    bc = t // inH
    dy = np.asarray(dy, F32)
    acc = np.zeros(n, F32)
    for sh in range(sH):
        for sw in range(sW):
            ho, wo = h * sH + sh, w * sW + sw
            ok = (ho < outH) & (wo < outW)
            src = np.where(ok, (bc * outH + ho) * outW + wo, 0)
            acc = np.where(ok, (acc + dy[src]).astype(F32), acc)
    return acc


def _channel_map(batch, c_in, spatial, c_out, c_off, limit):
    n = batch * c_in * spatial if limit is None else min(batch * c_in * spatial, limit)
    i = np.arange(n, dtype=np.int64)
    s = i % spatial
    t = i // spatial
    c = t % c_in
    b = t // c_in
    return i, (b * c_out + c + c_off) * spatial + s


def concat_insert(out, x, batch, c_in, spatial, c_out, c_off, limit=None):
    """nn_concat_insert.hlsl:12-27: Out[b, c + c_off, s] = X[b, c, s] (in place on `out`)."""
    i, dst = _channel_map(batch, c_in, spatial, c_out, c_off, limit)
    out[dst] = np.asarray(x, F32)[i]
    return out


def slice_channels(dy, batch, c_in, spatial, c_out, c_off, limit=None):
    """nn_slice.hlsl:12-27: DX[b, c, s] = DY[b, c + c_off, s] for flat index < limit."""
    _, src = _channel_map(batch, c_in, spatial, c_out, c_off, limit)
    return np.asarray(dy, F32)[src]


def maxpool_forward(x, batch, inC, inH, inW, p, stride, outH, outW, lim_w=None, lim_h=None, lim_bc=None):
    """nn_maxpool_forward.hlsl:16-52: per output (bc, oh, ow) the window
    [oh*stride, +p) x [ow*stride, +p), clipped to the input, scanned rows outer /
    columns inner with a strict `>` from -1e30 (first maximum wins; NaN never
    selected); the index is the flat input index, 0xFFFFFFFF when nothing beat
    -1e30.  Returns (out_idx, values, indices) for the threads that run."""
    lw = outW if lim_w is None else min(outW, lim_w)
    lh = outH if lim_h is None else min(outH, lim_h)
    lb = batch * inC if lim_bc is None else min(batch * inC, lim_bc)
    bc, oh, ow = np.meshgrid(np.arange(lb, dtype=np.int64), np.arange(lh, dtype=np.int64),
                             np.arange(lw, dtype=np.int64), indexing="ij")
    x = np.asarray(x, F32)
    best = np.full(bc.shape, F32(-1e30), F32)
    idx = np.full(bc.shape, NO_INDEX, np.uint32)
    base = bc * (inH * inW)
    for ph in range(p):
        for pw in range(p):
            ih, iw = oh * stride + ph, ow * stride + pw
            ok = (ih < inH) & (iw < inW)
            src = np.where(ok, base + ih * inW + iw, 0)
            v = x[src]
            upd = ok & (v > best)
            best = np.where(upd, v, best)
            idx = np.where(upd, src.astype(np.uint32), idx)
    out_idx = bc * (outH * outW) + oh * outW + ow
    return out_idx.ravel(), best.ravel(), idx.ravel()


def maxpool_backward(dinput, dz, indices_bits, batch, inC, outH, outW, lim_w=None, lim_h=None, lim_bc=None):
    """nn_maxpool_backward.hlsl:12-25: dInput[idx[o]] = dZ[o] for every output o
    that runs and whose index is not 0xFFFFFFFF (in place; other elements keep
    their value).  Indices past the buffer are dropped, as D3D11 drops
    out-of-range UAV writes.  Two outputs naming one element (overlapping
    windows) leave either value in the reference; callers of this oracle use
    windows that do not overlap."""
    lw = outW if lim_w is None else min(outW, lim_w)
    lh = outH if lim_h is None else min(outH, lim_h)
    lb = batch * inC if lim_bc is None else min(batch * inC, lim_bc)
    bc, oh, ow = np.meshgrid(np.arange(lb, dtype=np.int64), np.arange(lh, dtype=np.int64),
                             np.arange(lw, dtype=np.int64), indexing="ij")
    o = (bc * (outH * outW) + oh * outW + ow).ravel()
    tgt = np.asarray(indices_bits, np.uint32)[o].astype(np.int64)
    ok = (tgt != int(NO_INDEX)) & (tgt < dinput.size)
    dinput[tgt[ok]] = np.asarray(dz, F32)[o[ok]]
    return dinput


def conv_reshape(mm, bias, batch, OC, OH, OW, act, lim_bp=None, lim_oc=None):
    """nn_conv_reshape.hlsl:13-30: z = mm[oc, b*OH*OW + pixel] + bias[oc] (fp32),
    act 1 -> max(0, z), act 2 -> tanh(z), else z; stored NCHW at
    [b, oc, pixel].  Returns (dst, values)."""
    P = OH * OW
    BP = batch * P
    lbp = BP if lim_bp is None else min(BP, lim_bp)
    loc = OC if lim_oc is None else min(OC, lim_oc)
    oc, bp = np.meshgrid(np.arange(loc, dtype=np.int64), np.arange(lbp, dtype=np.int64), indexing="ij")
    z = (np.asarray(mm, F32)[oc * BP + bp] + np.asarray(bias, F32)[oc]).astype(F32)
    if act == 1:
        a = _relu(z)
    elif act == 2:
        a = np.tanh(z.astype(F64)).astype(F32)
    else:
        a = z
    dst = (bp // P) * (OC * P) + oc * P + bp % P
    return dst.ravel(), a.ravel()


def conv_grad_reshape(dz, batch, outC, outH, outW, fwd=None, lim_bp=None, lim_oc=None):
    """nn_conv_grad_reshape.hlsl:16-28 (and nn_conv_grad_reshape_relu.hlsl:21-39 when
    `fwd` is given): out[oc, b*P + pixel] = dZ[b, oc, pixel], zeroed where the
    forward output is <= 0 (NaN keeps the gradient).  Returns (dst, values)."""
    P = outH * outW
    BP = batch * P
    lbp = BP if lim_bp is None else min(BP, lim_bp)
    loc = outC if lim_oc is None else min(outC, lim_oc)
    oc, bp = np.meshgrid(np.arange(loc, dtype=np.int64), np.arange(lbp, dtype=np.int64), indexing="ij")
    src = (bp // P) * (outC * P) + oc * P + bp % P
    g = np.asarray(dz, F32)[src]
    if fwd is not None:
        g = np.where(np.asarray(fwd, F32)[src] <= 0, F32(0.0), g).astype(F32)
    return (oc * BP + bp).ravel(), g.ravel()


def cb_words(cb: bytes, n: int = 16):
    """Decode up to `n` little-endian u32 cbuffer words (missing words read 0)."""
    cb = bytes(cb or b"")
    cb = cb + b"\x00" * max(0, 4 * n - len(cb))
    return list(struct.unpack("<%dI" % n, cb[: 4 * n]))


def run_shader(name: str, srvs, uavs, groups, cb: bytes) -> None:
    """Execute shader `name` in place on NumPy buffers, like `RunShader` (engine.cpp:396-400).

    `srvs`/`uavs` are lists of flat float32 arrays (views are written in place).
    Unknown names are ignored, as the reference does (engine.cpp:397-399).
    """
    u = cb_words(cb)
    g = tuple(int(v) for v in groups)
    if name == "add_bias" or name == "bias_relu":
        M, N = u[0], u[1]
        fn = add_bias if name == "add_bias" else bias_relu
        r = fn(srvs[0], srvs[1], M, N, limit=g[0] * 256)
        uavs[0][: r.size] = r
    elif name == "relu":
        n = min(uavs[0].size, g[0] * 256)
        uavs[0][:n] = relu(srvs[0], n)
    elif name == "relu_grad":
        n = _lim(u[0], g)
        uavs[0][:n] = relu_grad(srvs[0], srvs[1], n)
    elif name == "relu6":
        n = _lim(u[0], g)
        uavs[0][:n] = relu6(srvs[0], n)
    elif name == "relu6_grad":
        n = _lim(u[0], g)
        uavs[0][:n] = relu6_grad(srvs[0], srvs[1], n)
    elif name == "leaky_relu":
        n = _lim(u[0], g)
        uavs[0][:n] = leaky_relu(srvs[0], n, u2f(u[1]))
    elif name == "leaky_relu_grad":
        n = _lim(u[0], g)
        uavs[0][:n] = leaky_relu_grad(srvs[0], srvs[1], n, u2f(u[1]))
    elif name == "sigmoid":
        n = _lim(u[0], g)
        uavs[0][:n] = sigmoid_f64(srvs[0], n)
    elif name == "sigmoid_grad":
        n = _lim(u[0], g)
        uavs[0][:n] = sigmoid_grad(srvs[0], srvs[1], n)
    elif name == "add":
        n = _lim(u[0] * u[1], g)
        uavs[0][:n] = add(srvs[0], srvs[1], n, 1)
    elif name == "scale_add":
        n = _lim(u[0], g)
        uavs[0][:n] = scale_add(srvs[0], srvs[1], n, u2f(u[1]), u2f(u[2]))
    elif name == "grad_accum":
        n = _lim(u[0], g)
        uavs[0][:n] = grad_accum(uavs[0], srvs[0], n)
    elif name == "bias_grad":
        k = min(u[1], g[0])
        uavs[0][:k] = bias_grad(srvs[0], u[0], u[1], u[2], u[3], limit=k)
    elif name == "global_avg_pool":
        k = min(u[0] * u[1], g[0])
        uavs[0][:k] = global_avg_pool(srvs[0], u[0], u[1], u[2], limit=k)
    elif name == "global_avg_pool_backward":
        n = _lim(u[0] * u[1] * u[2], g)
        uavs[0][:n] = global_avg_pool_backward(srvs[0], u[0], u[1], u[2])[:n]
    elif name == "softmax":
        b = min(u[0], g[0] * 16)
        uavs[0][: b * u[1]] = softmax_f64(srvs[0], u[0], u[1], limit=b).ravel()
    elif name == "loss":
        uavs[0][0] = ce_loss_f64(srvs[0], srvs[1], u[0], u[1])
    elif name == "softmax_ce_grad":
        B, K = u[0], u[1]
        kx, by = min(K, g[0] * 16), min(B, g[1] * 16)
        r = softmax_ce_grad(srvs[0], srvs[1], B, K, kx, by)
        view = uavs[0][: B * K].reshape(B, K)
        view[:by, :kx] = r
    elif name == "argmax_correct":
        cnt = argmax_correct(srvs[0], srvs[1], u[0], u[1], limit=g[0] * 256)
        bits = uavs[0].view(np.uint32)
        bits[0] = np.uint32((int(bits[0]) + cnt) & 0xFFFFFFFF)
    elif name == "accumulate_scalar":
        uavs[0][0] = accumulate_scalar(uavs[0], srvs[0])
    elif name == "rms":
        uavs[0][0] = rms(srvs[0], u[0])
    elif name == "grad_sq_reduce":
        count, off = u[0], u[1]
        k = g[0]
        uavs[0][off: off + k] = grad_sq_reduce(srvs[0], count, k)
    elif name == "grad_norm_final":
        norm, scale = grad_norm_final(srvs[0], u[0], u2f(u[1]))
        uavs[0][0] = norm
        uavs[0][1] = scale
    elif name == "sgd":
        n = _lim(u[0], g)
        uavs[0][:n] = sgd(uavs[0], srvs[0], n, u2f(u[1]), u2f(u[2]))
    elif name == "sgd_clipped":
        n = _lim(u[0], g)
        uavs[0][:n] = sgd_clipped(uavs[0], srvs[0], n, u2f(u[1]), srvs[1][1])
    elif name == "adam":
        n = _lim(u[0], g)
        w, m, v = adam(uavs[0], uavs[1], uavs[2], srvs[0], n, u2f(u[1]), u2f(u[2]),
                       u2f(u[3]), u2f(u[4]), u2f(u[5]), u2f(u[6]))
        uavs[0][:n], uavs[1][:n], uavs[2][:n] = w, m, v
    elif name == "batchnorm_mean_var":
        N, C, S, training, mom = u[0], u[1], u[2], u[3], u2f(u[4])
        c = min(C, g[0])
        mean, var = batchnorm_mean_var(srvs[0], N, C, S)
        uavs[0][:c] = mean[:c].astype(F32)
        uavs[1][:c] = var[:c].astype(F32)
        if training == 1:
            rm, rv = batchnorm_running(uavs[2][:c], uavs[3][:c], mean[:c], var[:c], N, S, mom)
            uavs[2][:c], uavs[3][:c] = rm, rv
    elif name == "batchnorm_forward":
        N, C, S, eps = u[0], u[1], u[2], u2f(u[3])
        n = _lim(N * C * S, g)
        uavs[0][:n] = batchnorm_forward(srvs[0], srvs[1], srvs[2], srvs[3], srvs[4],
                                        N, C, S, eps)[:n]
    elif name == "batchnorm_backward_reduce":
        N, C, S, eps = u[0], u[1], u[2], u2f(u[3])
        c = min(C, g[0])
        dg, db = batchnorm_backward_reduce(srvs[0], srvs[1], srvs[2], srvs[3], N, C, S, eps)
        uavs[0][:c], uavs[1][:c] = dg[:c], db[:c]
    elif name == "batchnorm_backward_dx":
        N, C, S, eps = u[0], u[1], u[2], u2f(u[3])
        n = _lim(N * C * S, g)
        uavs[0][:n] = batchnorm_backward_dx(srvs[0], srvs[1], srvs[2], srvs[3], srvs[4],
                                            srvs[5], srvs[6], N, C, S, eps)[:n]
    elif name == "dice_loss":
        b = min(u[0], g[0])
        uavs[0][:b] = dice_loss(srvs[0], srvs[1], u[0], u[1])[:b]
    elif name == "dice_loss_sums":
        b = min(u[0], g[0])
        uavs[0][: 3 * b] = dice_sums(srvs[0], srvs[1], u[0], u[1])[:b].astype(F32).ravel()
    elif name == "dice_loss_grad":
        n = _lim(u[0] * u[1], g)
        uavs[0][:n] = dice_loss_grad(srvs[0], srvs[1], srvs[2], u[0], u[1])[:n]
    elif name == "upsample":
        uavs[0][: _lim(u[0] * u[1] * u[4] * u[5], g)] = upsample(srvs[0], *u[:8], limit=g[0] * 256)
    elif name == "upsample_backward":
        r = upsample_backward(srvs[0], *u[:8], limit=g[0] * 256)
        uavs[0][: r.size] = r
    elif name == "concat_insert":
        concat_insert(uavs[0], srvs[0], *u[:5], limit=g[0] * 256)
    elif name == "slice":
        r = slice_channels(srvs[0], *u[:5], limit=g[0] * 256)
        uavs[0][: r.size] = r
    elif name == "maxpool_forward":
        o, v, i = maxpool_forward(srvs[0], *u[:8], lim_w=g[0] * 16, lim_h=g[1] * 16, lim_bc=g[2])
        uavs[0][o] = v
        uavs[1].view(np.uint32)[o] = i
    elif name == "maxpool_backward":
        maxpool_backward(uavs[0], srvs[0], srvs[1].view(np.uint32), *u[:4],
                         lim_w=g[0] * 16, lim_h=g[1] * 16, lim_bc=g[2])
    elif name == "conv_reshape":
        dst, v = conv_reshape(srvs[0], srvs[1], *u[:5], lim_bp=g[0] * 16, lim_oc=g[1] * 16)
        uavs[0][dst] = v
    elif name in ("conv_grad_reshape", "conv_grad_reshape_relu"):
        fwd = srvs[1] if name == "conv_grad_reshape_relu" else None
        dst, v = conv_grad_reshape(srvs[0], u[0], u[4], u[7], u[8], fwd=fwd, lim_bp=g[0] * 16, lim_oc=g[1] * 16)
        uavs[0][dst] = v
    # any other name: silently ignored, like engine.cpp:397-399


#: Reference shader names the CUDA library implements (the hot path).
HOT_PATH_SHADERS = (
    "add_bias", "bias_relu", "relu", "relu_grad", "relu6", "relu6_grad",
    "leaky_relu", "leaky_relu_grad", "sigmoid", "sigmoid_grad", "add",
    "scale_add", "grad_accum", "bias_grad", "global_avg_pool",
    "global_avg_pool_backward", "softmax", "loss", "softmax_ce_grad",
    "argmax_correct", "accumulate_scalar", "rms", "grad_sq_reduce",
    "grad_norm_final", "sgd", "sgd_clipped", "adam", "batchnorm_mean_var",
    "batchnorm_forward", "batchnorm_backward_reduce", "batchnorm_backward_dx",
    "dice_loss", "dice_loss_sums", "dice_loss_grad",
    "upsample", "upsample_backward", "concat_insert", "slice", "maxpool_forward",
    "maxpool_backward", "conv_reshape", "conv_grad_reshape", "conv_grad_reshape_relu",
)
