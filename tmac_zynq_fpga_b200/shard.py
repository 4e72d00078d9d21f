"""Vocab-row sharding of the tied-embedding logits GEMV across GPUs.

Each rank owns rows [r0, r1) of the 151936 x 896 Q8_0 matrix (contiguous,
151936 / world rows), computes its logits shard and the top-1 key of the shard
(tmac_gemv_top1, index_base = r0), and one int64 MAX all-reduce of that key
gives every rank the global greedy token.  The key layout is top1_key in
csrc/common.cuh: order-preserving float bits << 31 | (0x7FFFFFFF - index).
"""
from __future__ import annotations

import numpy as np


def shard_bounds(rows: int, world: int, rank: int):
    """Contiguous row range of `rank` (sizes differ by at most one row)."""
    return rank * rows // world, (rank + 1) * rows // world


def pack_keys(y: np.ndarray, index_base: int = 0) -> np.ndarray:
    """Host version of the device key, one per element of y (for checks)."""
    u = np.ascontiguousarray(y, dtype=np.float32).view(np.uint32).astype(np.uint64)
    neg = (u & 0x80000000) != 0
    ordered = np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    idx = np.arange(y.size, dtype=np.uint64) + np.uint64(index_base)
    return ((ordered << np.uint64(31)) | (np.uint64(0x7FFFFFFF) - idx)).astype(np.int64)


def unpack_key(key: int):
    """(value, index) of a key."""
    key = int(key)
    u = (key >> 31) & 0xFFFFFFFF
    u = (u & 0x7FFFFFFF) if (u & 0x80000000) else (~u & 0xFFFFFFFF)
    return float(np.array([u], np.uint32).view(np.float32)[0]), 0x7FFFFFFF - (key & 0x7FFFFFFF)


def top1_index(y: np.ndarray) -> int:
    """Lowest index among the largest values (the key's tie rule)."""
    return int(np.argmax(y))  # numpy returns the first maximum


def all_reduce_top1(key_tensor, group=None):
    """Merges per-rank keys (int64 tensor) in place with a MAX all-reduce."""
    import torch.distributed as dist
    dist.all_reduce(key_tensor, op=dist.ReduceOp.MAX, group=group)
    return key_tensor


def gather_logits(local, rows: int, out=None, group=None):
    """The full logits vector on every rank from each rank's vocab shard
    (get_logits_q8 returns all rows, sim/tmac_gguf.cpp:1820-1845): one
    all-gather of the shards, padded to the largest shard.  `local` is this
    rank's shard (a torch tensor on the process group's device, float32);
    returns (and fills `out`, if given) a float32 tensor [rows]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    most = -(-rows // world)
    if local.numel() == most:
        buf = local.contiguous()
    else:
        buf = torch.zeros(most, dtype=torch.float32, device=local.device)
        buf[: local.numel()] = local
    flat = torch.empty(world * most, dtype=torch.float32, device=local.device)
    dist.all_gather_into_tensor(flat, buf, group=group)
    if out is None:
        out = torch.empty(rows, dtype=torch.float32, device=local.device)
    if all(shard_bounds(rows, world, r)[1] - shard_bounds(rows, world, r)[0] == most for r in range(world)):
        out.copy_(flat[:rows])
    else:
        parts = flat.view(world, most)
        for r in range(world):
            r0, r1 = shard_bounds(rows, world, r)
            out[r0:r1] = parts[r, : r1 - r0]
    return out


def device_view(ptr: int, n: int):
    """A float32 CUDA tensor over n floats at device address ptr (no copy)."""
    import torch

    class _View:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (int(ptr), False), "version": 3}
    return torch.as_tensor(_View(), device="cuda")


# ------------------------------------------------------------------ prefill
# The multi-sequence prefill batch shards by sequence: rank r prefills sequences
# [s0, s1) of the batch with tmac_model_prefill on its own GPU.  Sequences are
# independent, so there is no collective on the data path; the per-sequence
# next tokens are gathered once at the end.

def sequence_shard(n_seq: int, world: int, rank: int):
    """Contiguous sequence range of `rank` (sizes differ by at most one)."""
    return shard_bounds(n_seq, world, rank)


def gather_next_tokens(local, n_seq: int, group=None):
    """All ranks' next tokens (int32 [s1 - s0] each) in batch order, on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    most = -(-n_seq // world)
    buf = torch.full((most,), -1, dtype=torch.int64, device=dev)
    buf[: len(local)] = torch.as_tensor(np.asarray(local, dtype=np.int64), device=dev)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    out = []
    for r in range(world):
        s0, s1 = sequence_shard(n_seq, world, r)
        out.append(parts[r][: s1 - s0].cpu().numpy())
    return np.concatenate(out).astype(np.int32)


# ------------------------------------------------ peer-memory top-1 exchange
class PeerTop1:
    """Global top-1 key over NVLink peer memory (tmac_xchg_*): every rank
    stores its shard key into every rank's exchange buffer and takes the
    maximum of this step's keys, in one small kernel per step, or inside the
    logits GEMV itself (gemv_top1).  Setup shares
    the CUDA IPC handles of the buffers over the process group."""

    def __init__(self, device: int, group=None, vocab: int = 0):
        import ctypes
        import torch.distributed as dist
        from . import lib, check, _P
        self._lib = lib()
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.handle = _P()
        self.vocab = int(vocab)
        f = self._lib.tmac_xchg_create_logits
        f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.POINTER(_P)]
        check(f(device, world, rank, self.vocab, ctypes.byref(self.handle)))
        buf = (ctypes.c_uint8 * 64)()
        check(self._lib.tmac_xchg_ipc_handle(self.handle, buf))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(buf), group=group)
        joined = b"".join(handles)
        check(self._lib.tmac_xchg_open(self.handle, joined))
        dist.barrier(group=group)

    def __call__(self, key_tensor, stream=None):
        from . import check
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(self._lib.tmac_xchg_top1(self.handle, key_tensor.data_ptr(), s))
        return key_tensor

    def gemv_top1(self, weight, x, y, key_tensor, index_base: int, stream=None):
        """Logits of this rank's vocab shard (batch 1) and the global top-1 key
        in one launch (tmac_xchg_gemv_top1: the exchange runs in the Q8_0
        GEMV's last CTA)."""
        from . import check
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(self._lib.tmac_xchg_gemv_top1(self.handle, weight.handle, x.data_ptr(), y.data_ptr(),
                                            key_tensor.data_ptr(), int(index_base), s))
        return key_tensor

    def logits(self):
        """This rank's full logits vector of the last step (created with vocab > 0;
        tmac_xchg_logits) as a float32 CUDA tensor viewing the exchange buffer:
        valid until the next exchange call."""
        import ctypes
        import torch
        from . import check
        p = ctypes.c_void_p()
        f = self._lib.tmac_xchg_logits
        f.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        check(f(self.handle, ctypes.byref(p)))
        return device_view(p.value, self.vocab)

    def free(self):
        if getattr(self, "handle", None):
            self._lib.tmac_xchg_free(self.handle)
            self.handle = None
