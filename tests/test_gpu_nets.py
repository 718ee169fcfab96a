"""BASELINE configs 3 and 5 (ResNet-50 and MobileNetV2 conv stacks) at batch 2: every layer, on
whatever kernel it dispatches to, equals the CPU oracle bit for bit (int8 requantized outputs)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("net", ["resnet50", "mobilenetv2"])
def test_network_layers_match_oracle(cuda_lib, net):
    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import nets

    specs = nets.NETS[net]()
    data = nets.NetData(specs, batch=2, seed=42, device=torch.device("cuda"))
    paths = {}
    for i in range(len(specs)):
        data.run_layer(i)
        paths.setdefault(b2q.last_path(), []).append(specs[i].name)
    torch.cuda.synchronize()
    assert "cuda-core-generic" not in paths, paths.get("cuda-core-generic")
    for i, sp in enumerate(specs):
        x, w, b, s = nets.host_layer_tensors(sp, i, 42, 0, 2)
        np.testing.assert_array_equal(data.layers[i][1].cpu().numpy(), x, err_msg=f"{sp.name} input")
        a = oracle.conv_args(2, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.pad, sp.pad, sp.stride, sp.stride, 1, 1,
                             sp.groups)
        acc = oracle.conv_s8(a, x, w, threads=2)
        e = sp.epilogue()
        ref = oracle.requant_s8(acc, b, s, e.zp_out, e.clamp_lo, e.clamp_hi)
        np.testing.assert_array_equal(data.layers[i][5].cpu().numpy(), ref, err_msg=sp.name)


def _epi_bounds(sp):
    from my_own_cnn_b200 import nets

    if sp.linear:
        return -128, 127
    return (0, nets.Q6) if sp.relu6 else (0, 127)


@pytest.mark.parametrize("net", ["resnet50", "mobilenetv2"])
def test_chained_network_matches_oracle(cuda_lib, net):
    """The whole int8 network chained on the device (residual adds fused into the conv epilogues,
    max / average pools) against the same chain run by the CPU oracle, one image."""
    from my_own_cnn_b200 import nets, synth

    seed = 31
    model = nets.ChainedNet(net, seed, "cuda")
    x = synth.fill_s8_table(torch.empty((1, 224, 224, 3), dtype=torch.int8, device="cuda"), seed, 1,
                            torch.from_numpy(nets.act_table()).cuda())
    y = model.forward(x)
    torch.cuda.synchronize()
    bufs = {0: synth.s8_table_host(seed, 1, nets.act_table(), 0, 224 * 224 * 3).reshape(1, 224, 224, 3)}
    for op in model.plan:
        src = bufs[op.src]
        if op.kind == "conv":
            sp = model.specs[op.layer]
            _, w, b, s = nets.host_layer_tensors(sp, op.layer, seed, 0, 1)
            a = oracle.conv_args(1, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.pad, sp.pad, sp.stride, sp.stride,
                                 groups=sp.groups)
            acc = oracle.conv_s8(a, src, w, threads=8)
            lo, hi = _epi_bounds(sp)
            if op.res >= 0:
                bufs[op.dst] = oracle.requant_res_s8(acc, b, s, bufs[op.res], nets.RES_SCALE, 0, lo, hi)
            else:
                bufs[op.dst] = oracle.requant_s8(acc, b, s, 0, lo, hi)
        elif op.kind == "maxpool":
            bufs[op.dst] = oracle.maxpool_s8(src, 3, 3, 2, 2, 1, 1)
        else:
            bufs[op.dst] = oracle.global_avgpool_s8(src)
    want = bufs[model.plan[-1].dst]
    np.testing.assert_array_equal(y.cpu().numpy(), want)
    assert np.count_nonzero(want) > want.size // 8  # the synthetic network does not collapse to zeros
