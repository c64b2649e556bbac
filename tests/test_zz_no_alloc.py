"""lewm_sample_candidates_noalloc: candidate sampling with no device allocation.

The no-allocation entry point keeps its coloring matrix and Philox key in a
fixed scratch array inside the library instead of a context workspace. Its
candidates must equal those of lewm_sample_candidates for the same inputs.
Both run the same sampling kernel; the only difference is that the coloring
matrix is built on the device in double precision instead of on the host, so
the outputs agree to float32 rounding (rtol = atol = 1e-5, tighter than the
2e-3 the sampling tests allow against the numpy oracle).

This file is collected last so that the entry point also runs after every
other test has used the library in the same process.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from lewm_flash_b200 import _lib
from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
from lewm_flash_b200.runtime import PlanOptions, Runtime

RTOL = ATOL = 1e-5

# (beta, time_axis, action_block, clip, injected): raw-time colored (ncol 25),
# block-layout colored (ncol 5), raw time with block 1 (ncol 5), white, and
# injected noise with clipping. Consecutive cases change the scratch contents.
CASES = [
    (2.0, "raw", 5, False, False),
    (1.0, "raw", 5, True, False),
    (2.0, "block", 5, False, False),
    (2.0, "raw", 1, False, False),
    (0.0, "raw", 1, False, False),
    (0.0, "raw", 1, True, True),
]


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def noalloc_sample(opts, B, T, A, S, it, mean, std, noise=None, lo=None, hi=None, plan_index=0, device=0):
    out = torch.empty(B, S, T, A, device=f"cuda:{device}")
    pd = opts.to_c(B, T, 1, plan_index)
    st = _lib.lib().lewm_sample_candidates_noalloc(C.byref(pd), A, S, it, _ptr(mean), _ptr(std), _ptr(noise),
                                                   _ptr(lo), _ptr(hi), _ptr(out), device,
                                                   C.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    if st != 0:
        raise RuntimeError(f"status {st}: {_lib.lib().lewm_last_error(None).decode()}")
    return out


def _inputs(B, S, T, A, seed):
    g = torch.Generator().manual_seed(seed)
    mean = torch.randn(B, T, A, generator=g).cuda()
    std = (torch.rand(B, T, A, generator=g) * 1.5 + 0.1).cuda()
    noise = torch.randn(B, S, T, A, generator=g).cuda()
    lo = torch.full((A,), -0.8).cuda()
    hi = torch.full((A,), 0.8).cuda()
    return mean, std, noise, lo, hi


@pytest.mark.gpu
def test_noalloc_sampling_matches_context_entry_point_on_consecutive_calls():
    desc = ModelDesc()
    B, S, T, A = 3, 64, 5, desc.action_dim
    # No-allocation calls first, before any context exists in this process.
    got = []
    for i, (beta, axis, block, clip, inj) in enumerate(CASES):
        opts = PlanOptions(num_samples=S, topk=4, n_steps=1, beta=beta, time_axis=axis, action_block=block,
                           clip_actions=clip, seed=1000 + i)
        mean, std, noise, lo, hi = _inputs(B, S, T, A, i)
        pair = []
        for it in (3, 4):  # two calls in a row, same scratch
            pair.append(noalloc_sample(opts, B, T, A, S, it, mean, std, noise if inj else None,
                                       lo if clip else None, hi if clip else None, plan_index=7 + i).clone())
        got.append((opts, (mean, std, noise, lo, hi), pair))
    torch.cuda.synchronize()

    rt = Runtime(desc, synthetic_state_dict(desc, 0), "cuda:0")
    for (opts, (mean, std, noise, lo, hi), pair), case in zip(got, CASES):
        inj = case[4]
        for it, out in zip((3, 4), pair):
            want = rt.sample_candidates(opts, S, it, mean, std, noise if inj else None, lo, hi,
                                        plan_index=7 + CASES.index(case))
            torch.cuda.synchronize()
            np.testing.assert_allclose(out.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL,
                                       err_msg=f"case {case} iter {it}")
        # the two iterations draw different noise (white or colored cases)
        if not inj:
            assert not torch.equal(pair[0][:, 1:], pair[1][:, 1:])
    rt.sync()


@pytest.mark.gpu
def test_noalloc_sampling_repeats_after_context_use():
    desc = ModelDesc()
    B, S, T, A = 2, 40, 5, desc.action_dim
    opts = PlanOptions(num_samples=S, topk=4, n_steps=1, beta=2.0, time_axis="raw", action_block=5, seed=5)
    mean, std, _, _, _ = _inputs(B, S, T, A, 11)
    a = noalloc_sample(opts, B, T, A, S, 2, mean, std, plan_index=3).clone()
    b = noalloc_sample(opts, B, T, A, S, 2, mean, std, plan_index=3).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # Warm calls allocate no device memory: free bytes stay the same over repeated calls
    # (the output buffer is allocated before the measurement).
    out = torch.empty(B, S, T, A, device="cuda:0")
    pd = opts.to_c(B, T, 1, 3)
    stream = C.c_void_p(torch.cuda.current_stream(0).cuda_stream)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    for it in range(8):
        st = _lib.lib().lewm_sample_candidates_noalloc(C.byref(pd), A, S, it, _ptr(mean), _ptr(std), None, None, None,
                                                       _ptr(out), 0, stream)
        assert st == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0


def test_noalloc_rejects_sizes_beyond_the_scratch_limits():
    lib = _lib.lib()
    # horizon * action_dim = 13 * 10 = 130 > 128: rejected before any device work.
    pd = PlanOptions(num_samples=8, topk=4, n_steps=1, beta=2.0, action_block=5).to_c(1, 13, 1)
    dummy = C.c_void_p(16)
    st = lib.lewm_sample_candidates_noalloc(C.byref(pd), 10, 8, 0, dummy, dummy, None, None, None, dummy, 0, None)
    assert st == 2  # LEWM_UNSUPPORTED_SHAPE
    assert b"exceeds 128" in lib.lewm_last_error(None)
    pd = PlanOptions(num_samples=8, topk=4, n_steps=1, beta=2.0, action_block=3).to_c(1, 5, 1)
    st = lib.lewm_sample_candidates_noalloc(C.byref(pd), 10, 8, 0, dummy, dummy, None, None, None, dummy, 0, None)
    assert st == 1 and b"not divisible" in lib.lewm_last_error(None)
    st = lib.lewm_sample_candidates_noalloc(None, 10, 8, 0, dummy, dummy, None, None, None, dummy, 0, None)
    assert st == 1
    # horizon * action_dim = 2**20 * 2**12 wraps to 0 in 32-bit arithmetic; the check is 64-bit.
    pd = PlanOptions(num_samples=8, topk=4, n_steps=1).to_c(1, 1 << 20, 1)
    st = lib.lewm_sample_candidates_noalloc(C.byref(pd), 1 << 12, 8, 0, dummy, dummy, None, None, None, dummy, 0, None)
    assert st == 2 and b"exceeds 128" in lib.lewm_last_error(None)
