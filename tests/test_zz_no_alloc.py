"""The allocation-free global norm (r97b_global_norm_noalloc), called through the C ABI.

This entry point is for callers that cannot allocate device memory -- a host framework whose allocator
already owns the device, or a loop that cannot pay for cudaMalloc / cudaFree. It must give exactly what
r97b_global_norm gives with a caller-provided scratch buffer, on consecutive calls (the library's fixed
partials array keeps the previous call's contents, so a stale value would show on the second call), and it
must refuse an input larger than its fixed capacity without launching anything.

The file is named so that pytest collects it last."""
import ctypes

import numpy as np
import pytest
import torch

from r97training_b200._lib import lib

pytestmark = pytest.mark.gpu

R97B_ETOOLARGE = 4
MAX_ELEMS = 65536 * 4096


def _with_scratch(g, inv_k, max_norm):
    """The existing entry point, with its partials in a buffer this test allocates."""
    L = lib()
    n = g.numel()
    scratch = torch.empty(L.r97b_global_norm_scratch_bytes(n) // 8, dtype=torch.float64, device=g.device)
    out = torch.zeros(2, dtype=torch.float32, device=g.device)
    s = torch.cuda.current_stream().cuda_stream
    rc = L.r97b_global_norm(ctypes.c_void_p(g.data_ptr()), n, inv_k, max_norm, ctypes.c_void_p(scratch.data_ptr()),
                            ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(out.data_ptr() + 4), ctypes.c_void_p(s))
    assert rc == 0
    return out


def _no_alloc(g, inv_k, max_norm):
    out = torch.zeros(2, dtype=torch.float32, device=g.device)
    s = torch.cuda.current_stream().cuda_stream
    rc = lib().r97b_global_norm_noalloc(ctypes.c_void_p(g.data_ptr()), g.numel(), inv_k, max_norm,
                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(out.data_ptr() + 4),
                                        ctypes.c_void_p(s))
    assert rc == 0
    return out


def test_no_alloc_matches_scratch_version_on_two_calls(cuda):
    rs = np.random.RandomState(2024)
    # a large call, then a smaller one: the second must not see the first's partials
    for n, inv_k, max_norm, std in ((5_000_123, 1.0, 0.0, 1e-2), (300_001, 0.5, 0.25, 3e-2)):
        g = torch.from_numpy((rs.normal(size=n) * std).astype(np.float32)).to(cuda)
        want = _with_scratch(g, inv_k, max_norm)
        got = _no_alloc(g, inv_k, max_norm)
        torch.cuda.synchronize()
        w, o = want.cpu().numpy(), got.cpu().numpy()
        # the same kernels in the same order: identical bits (the bar of this repo's f32 reductions is
        # a relative 1e-6, which identical bits meet)
        assert np.array_equal(w.view(np.uint32), o.view(np.uint32)), (n, w, o)
        ref = np.float32(np.sqrt(np.sum((g.cpu().numpy().astype(np.float64) * inv_k) ** 2)))
        assert abs(float(o[0]) - float(ref)) <= 1e-6 * float(ref)


def test_no_alloc_calls_queued_back_to_back(cuda):
    """Three calls of different sizes queued on one stream with no host wait between them, each writing
    its own output slots, then one synchronise: stream order alone must keep each call's partials from
    the next call's, so every result equals the scratch version's bit for bit."""
    rs = np.random.RandomState(7)
    sizes = ((4_194_305, 1.0, 0.0), (65_537, 0.25, 1e-3), (1_048_576, 1.0, 0.5))
    gs = [torch.from_numpy((rs.normal(size=n) * 1e-2).astype(np.float32)).to(cuda) for n, _, _ in sizes]
    wants = [_with_scratch(g, k, c) for g, (_, k, c) in zip(gs, sizes)]
    torch.cuda.synchronize()
    out = torch.zeros(2 * len(sizes), dtype=torch.float32, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    for i, (g, (n, inv_k, max_norm)) in enumerate(zip(gs, sizes)):
        rc = lib().r97b_global_norm_noalloc(ctypes.c_void_p(g.data_ptr()), n, inv_k, max_norm,
                                            ctypes.c_void_p(out.data_ptr() + 8 * i),
                                            ctypes.c_void_p(out.data_ptr() + 8 * i + 4), ctypes.c_void_p(s))
        assert rc == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(len(sizes), 2)
    for i, w in enumerate(wants):
        assert np.array_equal(w.cpu().numpy().view(np.uint32), got[i].view(np.uint32)), (i, w, got[i])


def test_no_alloc_rejects_inputs_beyond_its_capacity(cuda):
    out = torch.zeros(2, dtype=torch.float32, device=cuda)
    g = torch.zeros(1, dtype=torch.float32, device=cuda)  # never read: the size check comes first
    rc = lib().r97b_global_norm_noalloc(ctypes.c_void_p(g.data_ptr()), MAX_ELEMS + 1, 1.0, 0.0,
                                        ctypes.c_void_p(out.data_ptr()), None, None)
    assert rc == R97B_ETOOLARGE
