"""Sharding of the hot path across the GPUs of one node.

One process per GPU.  The NCCL communicator belongs to libdct_cuda.so (its
dct_dist_* entry points); this module is the host side: the split of an axis
into contiguous shards, the exchange of the NCCL unique id over an existing
`torch.distributed` process group (any backend), and thin wrappers that pass
library buffer handles to the sharded ops.

The reference drives one D3D11 device and has no multi-GPU path
(engine.cpp:61-129); which op exchanges what:

  ============================  =====================================  ==========
  op                            shard                                  exchange
  ============================  =====================================  ==========
  elementwise / broadcast (C2)  rows of the output                     none
  axis -1 reductions (C3)       rows                                   none
  axis 0 reductions (C3)        rows (the reduced axis)                reduce()
  full reduction (C3)           contiguous slice                       reduce_all()
  softmax + CE (C4)             rows; global divisor                   softmax_ce()
  Adam (C5a)                    contiguous slice of the flat vector    none
  BatchNorm (C5b)               batch N                                batchnorm_*()
  ============================  =====================================  ==========

Every exchange gathers one small record per rank and folds them on the device
in rank order, so all ranks get identical results, and at world size 1 the
sharded ops are bit-identical to the single-GPU entry points.  The records
travel through NVLink peer memory when every rank could map every other (CUDA
IPC mappings set up at init; the op's last kernel stores its record words into
the peers as tagged lines, waits for theirs and folds), else by an NCCL
all-gather.

    import torch.distributed as td
    td.init_process_group("nccl")                 # or "gloo"
    comm = Communicator.from_process_group(timeout_s=60)
    off, cnt = shard_range(rows, comm.world, comm.rank)
    comm.reduce("sum", x, 1, cnt, cols, off, rows, out)
    comm.close()
"""
from __future__ import annotations

import ctypes as C

from . import _abi, load_library

__all__ = ["shard_range", "Communicator", "nccl_available"]


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Balanced contiguous split: shard `rank` of `n` items is [offset, offset + count).

    The first n % world shards hold one extra item.  Same rule as the library's
    dct_dist_shard."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"shard_range: need n >= 0 and 0 <= rank < world (n={n}, world={world}, rank={rank})")
    base, rem = divmod(n, world)
    count = base + (1 if rank < rem else 0)
    offset = rank * base + min(rank, rem)
    return offset, count


def _lib():
    """The library, after PyTorch (when installed) has loaded its own NCCL.

    libdct_cuda.so dlopens "libnccl.so.2" and takes an already-loaded copy
    first; importing torch beforehand makes that copy the one PyTorch links, so
    one process never holds two NCCL builds under the same soname."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass
    return load_library()


def nccl_available() -> bool:
    return bool(_lib().dct_dist_available())


def _h(x):
    """A library buffer handle from a handle, an int, or an object with `.handle`."""
    if x is None:
        return None
    h = getattr(x, "handle", x)
    return h.value if isinstance(h, C.c_void_p) else h


class Communicator:
    """The library's NCCL communicator for this process (one per process)."""

    ID_BYTES = 128

    def __init__(self, rank: int, world: int, uid: bytes, timeout_s: float = 120.0):
        self.lib = _lib()
        self.rank, self.world = rank, world
        if len(uid) != self.ID_BYTES:
            raise ValueError("the NCCL unique id is 128 bytes")
        buf = C.create_string_buffer(uid, self.ID_BYTES)
        _abi.check(self.lib, self.lib.dct_dist_init(buf, self.ID_BYTES, world, rank, float(timeout_s)),
                   "dct_dist_init")
        self._open = True

    @classmethod
    def new_unique_id(cls) -> bytes:
        lib = _lib()
        buf = C.create_string_buffer(cls.ID_BYTES)
        _abi.check(lib, lib.dct_dist_unique_id(buf, cls.ID_BYTES), "dct_dist_unique_id")
        return buf.raw

    @staticmethod
    def exchange_id(group=None) -> tuple[int, int, bytes]:
        """Rank 0 makes the NCCL unique id; every rank receives it over the
        torch.distributed group.  Returns (rank, world, id)."""
        import torch.distributed as td
        rank, world = td.get_rank(group), td.get_world_size(group)
        uid = Communicator.new_unique_id() if rank == 0 else b""
        obj = [uid]
        td.broadcast_object_list(obj, src=0, group=group)
        return rank, world, obj[0]

    @classmethod
    def from_process_group(cls, timeout_s: float = 120.0, group=None) -> "Communicator":
        rank, world, uid = cls.exchange_id(group)
        return cls(rank, world, uid, timeout_s)

    @classmethod
    def single(cls, timeout_s: float = 120.0) -> "Communicator":
        """A one-rank communicator (no process group needed)."""
        return cls(0, 1, cls.new_unique_id(), timeout_s)

    # -- plumbing -------------------------------------------------------------
    @property
    def peer_exchange(self) -> bool:
        """True when records travel through mapped peer memory rather than NCCL."""
        return bool(self.lib.dct_dist_peer_active())

    def _check(self, rc: int, what: str) -> None:
        _abi.check(self.lib, rc, what)

    def close(self) -> None:
        if getattr(self, "_open", False):
            self._open = False
            self._check(self.lib.dct_dist_finalize(), "dct_dist_finalize")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def barrier(self) -> None:
        self._check(self.lib.dct_dist_barrier(), "dct_dist_barrier")

    def allreduce(self, buf, count: int, op: str = "sum") -> None:
        self._check(self.lib.dct_dist_allreduce(_h(buf), count, _abi.REDUCE[op]), "dct_dist_allreduce")

    def broadcast(self, buf, count: int, root: int = 0) -> None:
        self._check(self.lib.dct_dist_broadcast(_h(buf), count, root), "dct_dist_broadcast")

    # -- sharded ops ------------------------------------------------------------
    def reduce(self, op: str, x, outer: int, len_local: int, inner: int, len_offset: int, len_total: int, out,
               out_idx=None) -> None:
        """x viewed as [outer, len_local, inner] holds rows [len_offset, len_offset + len_local) of an axis
        of extent len_total; out (and out_idx) get the reduction over the whole axis on every rank."""
        self._check(self.lib.dct_dist_reduce(_abi.REDUCE[op], _h(x), outer, len_local, inner, len_offset, len_total,
                                             _h(out), _h(out_idx)), "dct_dist_reduce")

    def reduce_all(self, op: str, x, n_local: int, out, want_host: bool = False):
        v = C.c_double(0.0)
        self._check(self.lib.dct_dist_reduce_all(_abi.REDUCE[op], _h(x), n_local, _h(out),
                                                 C.byref(v) if want_host else None), "dct_dist_reduce_all")
        return v.value if want_host else None

    def softmax_ce(self, logits, labels, rows_local: int, K: int, probs=None, dlogits=None, loss=None,
                   logprobs=None, global_rows: int | None = None, labels_int32: bool = False) -> None:
        """Fused softmax + CE over this rank's rows; loss and dlogits use the global batch."""
        div = float(global_rows if global_rows is not None else rows_local)
        self._check(self.lib.dct_dist_softmax_ce(_h(logits), _h(labels), int(labels_int32), rows_local, K, _h(probs),
                                                 _h(dlogits), _h(loss), _h(logprobs), div, div),
                    "dct_dist_softmax_ce")

    def batchnorm_forward_train(self, x, gamma, beta, running_mean, running_var, batch_mean, batch_var, y,
                                N_local: int, C_: int, S: int, eps: float = 1e-5, momentum: float = 0.1) -> None:
        self._check(self.lib.dct_dist_batchnorm_forward_train(
            _h(x), _h(gamma), _h(beta), _h(running_mean), _h(running_var), _h(batch_mean), _h(batch_var), _h(y),
            N_local, C_, S, eps, momentum), "dct_dist_batchnorm_forward_train")

    def batchnorm_backward(self, x, dy, batch_mean, batch_var, gamma, dgamma, dbeta, dx, N_local: int, C_: int,
                           S: int, eps: float = 1e-5) -> None:
        self._check(self.lib.dct_dist_batchnorm_backward(
            _h(x), _h(dy), _h(batch_mean), _h(batch_var), _h(gamma), _h(dgamma), _h(dbeta), _h(dx), N_local, C_, S,
            eps), "dct_dist_batchnorm_backward")
