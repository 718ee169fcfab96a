"""The conv entry point that allocates nothing (b200q_conv2d_s8_packed_noalloc).

It exists for callers that may not allocate GPU memory themselves -- plugins whose host runtime
owns and budgets all device memory, or latency-critical code where a cudaMalloc is not allowed.
Its scratch is one fixed device array of the library, shared by all calls on a device.  This file
is collected last on purpose, so a run that stops at the first failure has run everything else.
The test calls the entry point twice in a row through the C ABI (the second call reuses the
scratch left by the first) and compares both results with b200q_conv2d_s8 and with the CPU oracle,
bit for bit.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from my_own_cnn_b200 import _lib
from tests.kat import rng_s8

pytestmark = pytest.mark.gpu


def _call(name, x, w, bias, scale, y, shape, params, epi):
    n, h, wd, c, r, s, k = shape
    cp = _lib.CConvParams(*params)
    ce = _lib.CEpilogue(*epi)
    ptr = lambda t: 0 if t is None else t.data_ptr()
    fn = getattr(_lib.lib(), name)
    return fn(ptr(x), ptr(w), ptr(bias), ptr(scale), ptr(y), n, h, wd, c, r, s, k, ctypes.byref(cp),
              ctypes.byref(ce), torch.cuda.current_stream().cuda_stream)


def _case(seed, shape, params, epi, out_dtype):
    n, h, wd, c, r, s, k = shape
    pad_h, pad_w, sh, sw, dh, dw, _ = params
    ho = (h + 2 * pad_h - dh * (r - 1) - 1) // sh + 1
    wo = (wd + 2 * pad_w - dw * (s - 1) - 1) // sw + 1
    x = torch.from_numpy(rng_s8(seed, (n, h, wd, c))).cuda()
    w = torch.from_numpy(rng_s8(seed + 1, (k, r, s, c))).cuda()
    rng = np.random.default_rng(seed + 2)
    bias = torch.from_numpy(rng.integers(-2**15, 2**15, size=k).astype(np.int32)).cuda()
    scale = torch.from_numpy(rng.uniform(1e-4, 1e-3, size=k).astype(np.float32)).cuda()
    mk = lambda: torch.empty((n, ho, wo, k), dtype=out_dtype, device="cuda")
    return dict(x=x, w=w, bias=bias, scale=scale, shape=shape, params=params, epi=epi, y_new=mk(), y_ref=mk())


def _oracle_out(cs):
    """The CPU oracle's result for a case (int32: accumulators + bias, int8: the requantized codes)."""
    from oracle import oracle

    n, h, wd, c, r, s, k = cs["shape"]
    pad_h, pad_w, sh, sw, dh, dw, groups = cs["params"]
    a = oracle.conv_args(n, h, wd, c, r, s, k, pad_h, pad_w, sh, sw, dh, dw, groups)
    acc = oracle.conv_s8(a, cs["x"].cpu().numpy(), cs["w"].cpu().numpy(), threads=4)
    bias = cs["bias"].cpu().numpy()
    kind, zp, lo, hi = cs["epi"]
    if kind == _lib.OUT_S32:
        return (acc.astype(np.int64) + bias).astype(np.uint32).astype(np.int32).reshape(cs["y_new"].shape)
    return oracle.requant_s8(acc, bias, cs["scale"].cpu().numpy(), zp, lo, hi).reshape(cs["y_new"].shape)


def test_noalloc_conv_matches_existing_entry_on_two_calls_in_a_row(cuda_lib):
    cases = [
        # MobileNetV2 stem (3x3/2, C = 3 -> 32), int8 requant with ReLU
        _case(7, (2, 128, 128, 3, 3, 3, 32), (1, 1, 2, 2, 1, 1, 1), (_lib.OUT_S8, 0, 0, 127), torch.int8),
        # ResNet-50 stem geometry (7x7/2, C = 3 -> 64), int32 accumulators + bias
        _case(11, (3, 64, 64, 3, 7, 7, 64), (3, 3, 2, 2, 1, 1, 1), (_lib.OUT_S32, 0, 0, 0), torch.int32),
        # M = 100 rows (one partial 128-row tile), K = 24 output channels (no 16-byte vector stores)
        _case(13, (1, 10, 10, 16, 3, 3, 24), (1, 1, 1, 1, 1, 1, 1), (_lib.OUT_S8, 0, -128, 127), torch.int8),
    ]
    for cs in cases:  # two no-alloc calls back to back; the second overwrites the shared scratch
        rc = _call("b200q_conv2d_s8_packed_noalloc", cs["x"], cs["w"], cs["bias"], cs["scale"], cs["y_new"],
                   cs["shape"], cs["params"], cs["epi"])
        assert rc == 0, _lib.lib().b200q_last_error()
    for cs in cases:
        rc = _call("b200q_conv2d_s8", cs["x"], cs["w"], cs["bias"], cs["scale"], cs["y_ref"], cs["shape"],
                   cs["params"], cs["epi"])
        assert rc == 0, _lib.lib().b200q_last_error()
    torch.cuda.synchronize()
    assert _lib.lib().b200q_device_error() == 0
    for cs in cases:
        assert torch.equal(cs["y_new"], cs["y_ref"])
        assert np.array_equal(cs["y_new"].cpu().numpy(), _oracle_out(cs))


def test_noalloc_conv_rejects_requests_beyond_its_scratch(cuda_lib):
    cap = int(_lib.lib().b200q_noalloc_scratch_bytes())
    assert cap == 32 << 20
    # 64 x 112 x 112 output rows x 32 bytes = 25.7 MB fits; 96 images (38.5 MB) does not
    big = _case(3, (96, 224, 224, 3, 3, 3, 32), (1, 1, 2, 2, 1, 1, 1), (_lib.OUT_S8, 0, -128, 127), torch.int8)
    rc = _call("b200q_conv2d_s8_packed_noalloc", big["x"], big["w"], big["bias"], big["scale"], big["y_new"],
               big["shape"], big["params"], big["epi"])
    assert rc == _lib.B200Q_ERR_INVALID_ARG
    assert b"maximum" in _lib.lib().b200q_last_error()


def test_noalloc_conv_leaves_device_memory_unchanged(cuda_lib):
    """After a first call (which looks up the array's address), further calls on another stream take
    no device memory: the free-memory figure of the device does not move.  The stream is created
    before the first figure is read: in a fresh process torch's first stream creation sets up its
    stream pool, which takes device memory of its own."""
    cs = _case(17, (2, 96, 96, 3, 3, 3, 32), (1, 1, 2, 2, 1, 1, 1), (_lib.OUT_S8, 0, 0, 127), torch.int8)
    args = (cs["x"], cs["w"], cs["bias"], cs["scale"], cs["y_new"], cs["shape"], cs["params"], cs["epi"])
    side = torch.cuda.Stream()
    assert _call("b200q_conv2d_s8_packed_noalloc", *args) == 0, _lib.lib().b200q_last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    with torch.cuda.stream(side):
        for _ in range(3):
            assert _call("b200q_conv2d_s8_packed_noalloc", *args) == 0, _lib.lib().b200q_last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_conv_rejects_filter_rows_beyond_the_packed_limit(cuda_lib):
    """round_up(R*S*C, 32) above 16384 (here 3x3x1824 -> 16416) is refused, like the packed path."""
    cs = _case(19, (1, 3, 3, 1824, 3, 3, 16), (1, 1, 1, 1, 1, 1, 1), (_lib.OUT_S32, 0, 0, 0), torch.int32)
    rc = _call("b200q_conv2d_s8_packed_noalloc", cs["x"], cs["w"], cs["bias"], cs["scale"], cs["y_new"],
               cs["shape"], cs["params"], cs["epi"])
    assert rc == _lib.B200Q_ERR_UNSUPPORTED
    assert b"16384" in _lib.lib().b200q_last_error()
