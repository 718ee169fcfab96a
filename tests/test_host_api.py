"""CPU tests of the host side: the C-ABI library loads and exports every declared symbol,
the reference shim exports the reference's own symbols, and the Python mirror of the
reference interface validates like src/conv_types.h.  No compute call needs a GPU here."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from my_own_cnn_b200 import _lib
from my_own_cnn_b200.conv import BlockConv2DParams, Conv2DParams, infer_block_conv_shape, infer_conv_shape
from my_own_cnn_b200.quant import (QuantizationParametersS5, QuantizationParametersU8, get_zero_point,
                                   is_supported_quantized_input, DataType)

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    text = (ROOT / "include" / "b200q.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(b200q_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 15
    for name in syms:
        assert hasattr(L, name), name
    assert syms == set(_lib.EXPORTED_SYMBOLS) | (syms - set(_lib.EXPORTED_SYMBOLS))


def test_conv_out_shape_through_c_abi_matches_python():
    L = _lib.lib()
    cases = [((1, 56, 56, 64), (3, 3, 64, 64), Conv2DParams()),
             ((2, 224, 224, 3), (7, 7, 3, 64), Conv2DParams(3, 3, 2, 2, 1, 1, 1)),
             ((1, 9, 7, 8), (3, 3, 2, 12), Conv2DParams(1, 1, 2, 2, 2, 2, 4))]
    for xs, ws, p in cases:
        sh = infer_conv_shape(xs, ws, p)
        ho, wo = ctypes.c_int(), ctypes.c_int()
        cp = p.to_c()
        rc = L.b200q_conv_out_shape(xs[1], xs[2], xs[3], ws[0], ws[1], ws[3], ctypes.byref(cp), ctypes.byref(ho),
                                    ctypes.byref(wo))
        assert rc == 0 and (ho.value, wo.value) == (sh.ho, sh.wo)


@pytest.mark.parametrize("xs,ws,p,msg", [
    ((1, 8, 8, 6), (3, 3, 3, 4), Conv2DParams(groups=0), "groups must be > 0"),
    ((1, 8, 8, 6), (3, 3, 1, 4), Conv2DParams(groups=4), "input channels must be divisible by groups"),
    ((1, 8, 8, 6), (3, 3, 3, 5), Conv2DParams(groups=2), "output channels must be divisible by groups"),
    ((1, 8, 8, 6), (3, 3, 2, 4), Conv2DParams(groups=2), "filter cin_per_group mismatch"),
    ((1, 2, 2, 4), (5, 5, 4, 4), Conv2DParams(pad_h=0, pad_w=0), "invalid output size (negative numerator)"),
    ((1, 8, 8, 4), (3, 3, 4, 4), Conv2DParams(stride_h=0), "stride must be > 0"),
])
def test_infer_conv_shape_errors_like_reference(xs, ws, p, msg):
    with pytest.raises(RuntimeError, match=re.escape(msg)):
        infer_conv_shape(xs, ws, p)


def test_c_abi_rejects_bad_shapes_with_status():
    L = _lib.lib()
    ho, wo = ctypes.c_int(), ctypes.c_int()
    bad = _lib.CConvParams(1, 1, 0, 1, 1, 1, 1)
    assert L.b200q_conv_out_shape(8, 8, 4, 3, 3, 4, ctypes.byref(bad), ctypes.byref(ho), ctypes.byref(wo)) == 1
    assert b"stride" in L.b200q_last_error()
    g0 = _lib.CConvParams(1, 1, 1, 1, 1, 1, 0)
    assert L.b200q_conv_out_shape(8, 8, 4, 3, 3, 4, ctypes.byref(g0), ctypes.byref(ho), ctypes.byref(wo)) == 1


def test_block_shape_checks():
    p = BlockConv2DParams(Conv2DParams(), 2, 3)
    sh = infer_block_conv_shape((2, 6, 6, 4), (5, 2, 3, 3, 3, 4), p)
    assert (sh.base.ho, sh.block_ho, sh.block_wo) == (6, 3, 2)
    with pytest.raises(RuntimeError, match="divisible by block grid"):
        infer_block_conv_shape((2, 5, 6, 4), (5, 2, 3, 3, 3, 4), p)
    with pytest.raises(RuntimeError, match="block grid mismatch"):
        infer_block_conv_shape((2, 6, 6, 4), (5, 3, 3, 3, 3, 4), p)


def test_qparams_layout_matches_reference_structs():
    # QuantizationParameters<LinQuantU8>: {uint8 zp; float scale; bool symmetric} -> 12 bytes
    assert ctypes.sizeof(QuantizationParametersU8) == 12
    assert QuantizationParametersU8.zero_point.offset == 0 and QuantizationParametersU8.scale.offset == 4
    # QuantizationParameters<LinQuantS5>: {int8 zp; uint8 n_bins; float scale} -> 8 bytes
    assert ctypes.sizeof(QuantizationParametersS5) == 8
    assert QuantizationParametersS5.scale.offset == 4
    assert get_zero_point(QuantizationParametersU8(200)) == 200
    assert get_zero_point(QuantizationParametersS5(-5, 31)) == -5
    assert is_supported_quantized_input(DataType.LinQuantU8) and not is_supported_quantized_input(DataType.Real32)


def test_reference_shim_exports_reference_symbols():
    shim = ROOT / "my_own_cnn_b200" / "libb200q_refshim.so"
    if not shim.exists():
        pytest.skip("shim is built only where the reference headers are present")
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    out = subprocess.run([nm, "-D", "-C", "--defined-only", str(shim)], capture_output=True, text=True).stdout
    for sym in ["conv_quant_detail::launch_fprop_nhwc_qi32_u8", "conv_quant_detail::launch_fprop_nhwc_qi32_s5",
                "conv_quant_detail::launch_block_fprop_nhwc_qi32_u8",
                "conv_quant_detail::launch_block_fprop_nhwc_qi32_s5", "bmm_matmul_i32"]:
        assert sym in out, sym


def test_product_package_does_not_import_oracle():
    """The product path never loads the CPU checker (build.py may compile it, nothing calls it)."""
    pat = re.compile(r"^\s*(import oracle|from oracle)|liboracle|libref_oracle", re.M)
    for f in (ROOT / "my_own_cnn_b200").rglob("*"):
        if f.suffix in (".py", ".cu", ".cuh", ".cpp", ".h") and f.name != "build.py":
            assert not pat.search(f.read_text()), f


@pytest.mark.parametrize("net,convs,residuals", [("resnet50", 53, 16), ("mobilenetv2", 52, 10)])
def test_chained_network_plans(net, convs, residuals):
    """The chained forward uses every conv of the layer table once, feeds each conv a buffer of its
    input shape, and adds a shortcut of the conv's output shape (host logic only)."""
    from my_own_cnn_b200 import nets

    specs = nets.NETS[net]()
    plan = nets.chain_plan(net)
    assert sorted(op.layer for op in plan if op.kind == "conv") == list(range(convs))
    assert sum(op.res >= 0 for op in plan) == residuals
    assert plan[-1].kind == "avgpool"
    shapes = {0: (224, 224, 3)}
    for op in plan:
        h, w, c = shapes[op.src]
        if op.kind == "conv":
            sp = specs[op.layer]
            assert (h, w, c) == (sp.h, sp.w, sp.c), sp.name
            ho, wo = sp.out_hw()
            shapes[op.dst] = (ho, wo, sp.k)
            if op.res >= 0:
                assert shapes[op.res] == shapes[op.dst], sp.name
        elif op.kind == "maxpool":
            shapes[op.dst] = ((h + 2 - 3) // 2 + 1, (w + 2 - 3) // 2 + 1, c)
        else:
            shapes[op.dst] = (1, 1, c)
    assert shapes[plan[-1].dst] == (1, 1, 2048 if net == "resnet50" else 1280)


def test_new_entry_points_validate_arguments():
    """Pool and residual entry points reject bad shapes with a status, before touching a GPU."""
    L = _lib.lib()
    assert L.b200q_maxpool_s8(None, None, 1, 8, 8, 16, 3, 3, 0, 2, 1, 1, None) == 1
    assert b"stride" in L.b200q_last_error()
    assert L.b200q_maxpool_s8(None, None, 1, 2, 2, 16, 5, 5, 1, 1, 4, 4, None) == 1
    assert L.b200q_global_avgpool_s8(None, None, 1, 0, 8, 16, None) == 1
    cp = _lib.CConvParams(0, 0, 1, 1, 1, 1, 1)
    ce = _lib.CEpilogue(1, 0, -128, 127)
    assert L.b200q_conv2d_s8_add(None, None, None, None, None, 1.0, None, 1, 8, 8, 16, 1, 1, 16,
                                 ctypes.byref(cp), ctypes.byref(ce), None) == 1
    assert b"residual" in L.b200q_last_error()


def test_conv_plan_dispatch_tables():
    """The host-side dispatch decision (b200q_conv2d_s8_plan, the same function the GPU dispatch
    uses) for the BASELINE workloads: network stems on space-to-depth row tiles, stride-1 3x3
    convs with C <= 128 on row tiles, other 3x3 convs on im2col, 1x1 convs tiled (config 4's long
    reduction on 2-SM tiles; narrow ones pixel-grouped: ResNet-50 s1b1.conv1, MobileNetV2
    g1b1.project / g2b1.expand / g2b1.project), depthwise on CUDA cores, C = 24 expands packed."""
    from collections import Counter

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import nets

    E, P = b2q.Epilogue, b2q.Conv2DParams
    assert b2q.conv2d_s8_plan(1, 56, 56, 64, 3, 3, 64, P(), E.int8()) == "tcgen05-rowtile"   # config 1 / smoke
    assert b2q.conv2d_s8_plan(512, 14, 14, 1024, 1, 1, 2048, P(0, 0), E.int8()) == "tcgen05-tiled"
    assert b2q.conv2d_s8_plan(512, 14, 14, 2048, 1, 1, 512, P(0, 0), E.int8()) == "tcgen05-tiled-2sm"
    want = {"resnet50": {"tcgen05-s2d": 1, "tcgen05-tiled": 32, "tcgen05-tiled-grouped": 1, "tcgen05-rowtile": 6,
                         "tcgen05-im2col": 13},
            "mobilenetv2": {"tcgen05-s2d": 1, "cuda-core-depthwise-tma": 17, "tcgen05-tiled": 29,
                            "tcgen05-tiled-grouped": 3, "tcgen05-packed": 2}}
    for net, batch in (("resnet50", 256), ("mobilenetv2", 512)):
        got = Counter(b2q.conv2d_s8_plan(batch, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.params(), sp.epilogue())
                      for sp in nets.NETS[net]())
        assert dict(got) == want[net], (net, dict(got))
    # residual adds never take the depthwise kernel; forced CUDA-core policy
    assert b2q.conv2d_s8_plan(2, 20, 20, 48, 3, 3, 48, P(groups=48), E.int8(), residual=True) == "cuda-core-generic"
    b2q.set_path_policy(1)
    try:
        assert b2q.conv2d_s8_plan(1, 56, 56, 64, 3, 3, 64, P(), E.int8()) == "cuda-core-generic"
        assert b2q.conv2d_s8_plan(2, 20, 20, 48, 3, 3, 48, P(groups=48), E.int8()) == "cuda-core-depthwise"
    finally:
        b2q.set_path_policy(0)
    with pytest.raises(RuntimeError, match="residual add needs int8"):
        b2q.conv2d_s8_plan(1, 8, 8, 16, 1, 1, 16, P(0, 0), E.int32(), residual=True)
