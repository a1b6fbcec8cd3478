"""Tensor-parallel GEMV + all-reduce over NVLink peer memory (host side).

TPComm wraps grout_tp_comm (include/grout_attn.h): the library allocates
this rank's receive/flag buffer (its own cudaMalloc, so the IPC handle maps
exactly that address), the handles are exchanged over a torch.distributed
process group (host objects only), and the peers' buffers are opened.  gemv_allreduce(w, x, residual, out) then computes, on every rank,
out = residual + sum over ranks of w_r @ x_r in one kernel (partials stored
directly into the peers' memory, per-block flags, bounded waits).  One
process per GPU; all ranks must issue the same calls in the same order.
"""
import ctypes

import torch

from . import attn


class TPComm:
    def __init__(self, rank, world, hidden, group=None, device=None):
        L = attn.lib()
        self.rank, self.world, self.hidden = rank, world, hidden
        self.comm = None
        handle = (ctypes.c_char * 64)()
        out = ctypes.c_void_p()
        attn._check(L.grout_tp_comm_create(world, hidden, ctypes.byref(out), handle))
        self.comm = out
        mine = bytes(handle)
        if world > 1:
            allh = [None] * world
            torch.distributed.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        blob = (ctypes.c_char * (64 * world)).from_buffer_copy(b"".join(allh))
        attn._check(L.grout_tp_comm_connect(self.comm, rank, blob))
        if world > 1:  # every rank has opened every buffer before anyone writes
            torch.distributed.barrier(group=group)

    def gemv_allreduce(self, w, x, out, residual=None):
        """out[hidden] = residual + all-reduce(w @ x); w [hidden, k] f16
        (this rank's shard), x [k] f16 (any leading dims of size 1)."""
        L = attn.lib()
        k = w.shape[1]
        attn._need(w.shape[0] == self.hidden and x.numel() == k and out.numel() == self.hidden,
                   "gemv_allreduce shape mismatch")
        attn._check(L.grout_gemv_allreduce(
            self.comm, ctypes.c_void_p(w.data_ptr()), k, ctypes.c_void_p(x.data_ptr()),
            ctypes.c_void_p(residual.data_ptr()) if residual is not None else None,
            ctypes.c_void_p(out.data_ptr()), attn._stream(x)))
        return out

    def allreduce(self, partial, out, residual=None):
        """out[hidden] = residual + all-reduce(partial); partial [hidden] f16."""
        L = attn.lib()
        attn._need(partial.numel() == self.hidden and out.numel() == self.hidden,
                   "allreduce shape mismatch")
        attn._check(L.grout_allreduce_residual(
            self.comm, ctypes.c_void_p(partial.data_ptr()),
            ctypes.c_void_p(residual.data_ptr()) if residual is not None else None,
            ctypes.c_void_p(out.data_ptr()), attn._stream(partial)))
        return out

    def close(self):
        if self.comm:
            attn.lib().grout_tp_comm_destroy(self.comm)
            self.comm = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
