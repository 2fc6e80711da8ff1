"""A bounded device wait that runs out ends cleanly: no fault, no hang, a
status the host reads, and a context that stays usable.

The fused row-parallel all-reduce is launched as rank 0 of a two-rank
exchange whose rank 1 never exists (both receive buffers are this GPU's own
memory, so nothing crosses to another device). Rank 0's CTAs store their
pieces into both buffers and then wait for rank 1's pieces, which nothing
writes: each wait gives up after about 2 s, raises device flag bit 0 and
lets the kernel return. The next ordinary launch on the same context is
exact, and the launch counter has advanced like any other launch's.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from helpers import MAX_REL_TOL, MEAN_REL_TOL, bf16_tensor, rel_errors, words_of
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu


def test_fused_allreduce_wait_gives_up_without_the_other_rank(oracle_mod):
    m, k, n = 256, 512, 8
    w = oracle_mod.llama_weight(m, k, seed=5)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    x = torch.randn(n, k, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    lib = runtime._cuda_library()
    rb, fb = ctypes.c_uint64(0), ctypes.c_uint64(0)
    runtime._check(lib.zipserv_mm_allreduce_sizes(m, n, 2, ctypes.byref(rb), ctypes.byref(fb)))
    recv = [torch.zeros(rb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    flags = [torch.zeros(max(fb.value, 16), dtype=torch.uint8, device="cuda") for _ in range(2)]
    state = torch.zeros(16, dtype=torch.uint8, device="cuda")
    y = torch.zeros(n, m, dtype=torch.bfloat16, device="cuda")
    recv_ptrs = (ctypes.c_void_p * 2)(*(t.data_ptr() for t in recv))
    flag_ptrs = (ctypes.c_void_p * 2)(*(t.data_ptr() for t in flags))
    torch.cuda.synchronize()
    assert runtime.device_flags() == 0

    start = time.monotonic()
    runtime._check(lib.zipserv_mm_allreduce(
        torch.cuda.current_stream().cuda_stream, *(b.data_ptr() for b in packed.buffers),
        packed.max_common, packed.max_rare, packed.start_exp, x.data_ptr(), y.data_ptr(),
        m, n, k, 2, 0, recv_ptrs, flag_ptrs, ctypes.c_void_p(state.data_ptr()), rb.value,
        fb.value))
    torch.cuda.synchronize()
    elapsed = time.monotonic() - start
    assert runtime.device_flags() & 1, "the wait for the missing rank did not report giving up"
    assert 1.0 < elapsed < 60.0, elapsed
    # The kernel's last CTA advanced this rank's launch counter as usual.
    assert int(state[:4].view(torch.int32).item()) == 1

    # Rank 0's own pieces reached its own buffer: the launch did its work up
    # to the exchange (the buffer is no longer all zeros).
    assert bool(recv[0].any())

    # The context is intact: an ordinary launch is exact and raises nothing.
    y2 = runtime.linear(x, packed)
    torch.cuda.synchronize()
    assert runtime.device_flags() == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = (x.float() @ bf16_tensor(w).cuda().float().t()).to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    mx, mean = rel_errors(words_of(y2), words_of(ref))
    assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (mx, mean)
    assert np.isfinite(y2.float().cpu().numpy()).all()
