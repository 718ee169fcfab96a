"""BASELINE configs 3 and 5 at the batch sizes the bench runs (ResNet-50 at 256, MobileNetV2 at 512):
the dispatch depends on the batch (e.g. small activations take the packed path), so every layer is
run at the benchmarked batch, its kernel family must equal the host-side plan for that batch, and
two deterministic images per layer (the first and the last of the batch) must equal the CPU oracle
bit for bit.  Also BASELINE config 2's per-column int8 output at full size (64 x 1024^3)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
BENCH_BATCH = {"resnet50": 256, "mobilenetv2": 512}


@pytest.mark.parametrize("net", ["resnet50", "mobilenetv2"])
def test_every_layer_at_benchmark_batch(cuda_lib, net):
    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import nets

    batch = BENCH_BATCH[net]
    seed = 42
    specs = nets.NETS[net]()
    threads = oracle.cpu_threads()
    for i, sp in enumerate(specs):
        # one layer at a time (tensor ids of layer i) keeps the footprint to one layer's tensors
        data = nets.NetData([sp], batch=batch, seed=seed, device=torch.device("cuda"), first_layer=i)
        data.run_layer(0)
        torch.cuda.synchronize()
        want = b2q.conv2d_s8_plan(batch, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.params(), sp.epilogue())
        assert b2q.last_path() == want, (sp.name, b2q.last_path(), want)
        assert b2q.last_path() != "cuda-core-generic", sp.name
        e = sp.epilogue()
        _, w, b, s = nets.host_layer_tensors(sp, i, seed, 0, 1)
        for img in (0, batch - 1):
            x, _, _, _ = nets.host_layer_tensors(sp, i, seed, img, 1)
            a = oracle.conv_args(1, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.pad, sp.pad, sp.stride, sp.stride, 1, 1,
                                 sp.groups)
            acc = oracle.conv_s8(a, x, w, threads=threads)
            ref = oracle.requant_s8(acc, b, s, e.zp_out, e.clamp_lo, e.clamp_hi)
            got = data.layers[0][5][img:img + 1].cpu().numpy()
            np.testing.assert_array_equal(got, ref, err_msg=f"{sp.name} image {img} ({b2q.last_path()})")
        del data
        torch.cuda.empty_cache()


def test_config2_int8_output_full_size_sampled(cuda_lib):
    """Config 2 (64 x 1024^3, NN) with the per-column requantized int8 output: sampled rows of three
    batch items against an exact int64 product requantized by the oracle."""
    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import synth

    batch, M, N, K = 64, 1024, 1024, 1024
    A = synth.fill_s8_uniform(torch.empty((batch, M, K), dtype=torch.int8, device="cuda"), 42, 101)
    B = synth.fill_s8_uniform(torch.empty((batch, K, N), dtype=torch.int8, device="cuda"), 42, 102)
    scale = synth.scales_f32(N, 42, 103)
    bias = synth.i32_uniform_host(42, 104, -2**15, 2**15, 0, N)
    C8 = b2q.bmm_s8(A, B, 0, 0, b2q.Epilogue.int8(), col_scale=torch.from_numpy(scale).cuda(),
                    bias=torch.from_numpy(bias).cuda())
    torch.cuda.synchronize()
    assert b2q.last_path() in ("tcgen05-tiled", "tcgen05-tiled-2sm")
    for bi in (0, 37, 63):
        Ah = synth.s8_uniform_host(42, 101, -127, 127, bi * M * K, M * K).reshape(M, K)
        Bh = synth.s8_uniform_host(42, 102, -127, 127, bi * K * N, K * N).reshape(K, N)
        rows = [0, 129, 640, 1023]
        acc = (Ah[rows].astype(np.int64) @ Bh.astype(np.int64)).astype(np.int32)
        np.testing.assert_array_equal(C8[bi, rows].cpu().numpy(), oracle.requant_s8(acc, bias, scale),
                                      err_msg=f"batch item {bi}")
