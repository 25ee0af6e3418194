"""Helpers shared by the GPU tests (not collected as tests)."""
from __future__ import annotations

import ctypes as C

import torch

from miniep_b200 import _lib, build
from miniep_b200.ep import Comm, EPMoEBackend, EPStats, Placement


def require_gpu():
    import pytest
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    build.build()


def world1_comm(E, topk, H, I, max_tokens, dtype):
    comm = Comm(num_layers=1, num_experts=E, topk=topk, hidden=H, inter=I, max_tokens=max_tokens,
                dtype=dtype, single_process=True, timeout_ms=5000)
    comm.install(Placement.naive(1, E, 1))
    return comm


def world1_backend(w_in, w_out, topk, max_tokens, stats=True, num_layers=1, force_simt=False,
                   single_cta=False):
    """A one-rank expert-parallel backend holding all experts of layer 0."""
    E, two_i, H = w_in.shape
    comm = Comm(num_layers=num_layers, num_experts=E, topk=topk, hidden=H, inter=two_i // 2,
                max_tokens=max_tokens, dtype=w_in.dtype, single_process=True, timeout_ms=5000)
    if force_simt:
        comm.set_option("force_simt", 1)
    if single_cta:
        comm.set_option("tc_single_cta", 1)
    placement = Placement.naive(num_layers, E, 1)
    comm.install(placement)
    st = EPStats(num_layers, E) if stats else None
    be = EPMoEBackend(0, comm, placement, list(range(E)), w_in.cuda(), w_out.cuda(), st)
    return be


class RawCtx:
    """Direct C-ABI context (no torch.distributed), for entry points tested
    in isolation."""

    def __init__(self, rank, world, layers, E, k, H, I, max_tokens, dtype):
        self.L = _lib.lib()
        self.ctx = C.c_void_p()
        code = _lib.MEP_BF16 if dtype == torch.bfloat16 else _lib.MEP_F32
        _lib.check(self.L.mep_ctx_create(rank, world, torch.cuda.current_device(), layers, E, k, H,
                                         I, max_tokens, code, 0, C.byref(self.ctx)), None)

    def call(self, name, *args):
        rc = getattr(self.L, name)(self.ctx, *args)
        _lib.check(rc, self.ctx, name)

    def rc(self, name, *args):
        return getattr(self.L, name)(self.ctx, *args)

    def close(self):
        self.L.mep_ctx_destroy(self.ctx)


def stream():
    return torch.cuda.current_stream().cuda_stream
