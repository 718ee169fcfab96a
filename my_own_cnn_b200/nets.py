"""Layer tables of the BASELINE network configurations and their seeded synthetic tensors.

Config 3, ResNet-50-shaped stack (224x224x3 NHWC input): stem 7x7/2 C3->64, then bottleneck blocks
(1x1 / 3x3 / 1x1, expansion 4) at 56/28/14/7 with widths 64/128/256/512 and 3/4/6/3 blocks, stride 2
on the 3x3 of the first block of stages 2-4, 1x1 projection shortcuts (stride 2 from stage 2).
Every conv: bias + ReLU requant epilogue to int8.

Config 5, MobileNetV2-shaped stack: stem 3x3/2 C3->32, inverted residual blocks
(t, c, n, s) = (1,16,1,1) (6,24,2,2) (6,32,3,2) (6,64,4,2) (6,96,3,1) (6,160,3,2) (6,320,1,1)
(expand 1x1 -> depthwise 3x3 -> project 1x1), then the final 1x1 320->1280.  ReLU6 is a clamp to
[0, q6] in the quantized domain with q6 = 96 (output scale 1/16: 6 / (1/16) = 96) on the stem,
expand, depthwise and final convs; the project convs are linear (clamp [-128, 127]).

Max-pool and the residual additions are not part of the conv path: every layer gets its own
synthetic input of the right shape (activations half-normal sigma 40 clipped to [0, 127], weights
normal sigma 30 clipped to [-127, 127], bias U[-2^15, 2^15], scales U[1e-4, 1e-3]).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import synth
from .conv import Conv2DParams, Epilogue, conv2d_s8_add_into, conv2d_s8_into, conv_out_shape
from .pool import global_avgpool_s8, maxpool_s8

Q6 = 96


@dataclass(frozen=True)
class LayerSpec:
    name: str
    h: int
    w: int
    c: int
    k: int
    r: int
    stride: int
    groups: int = 1
    relu6: bool = False
    linear: bool = False

    @property
    def pad(self) -> int:
        return self.r // 2

    def params(self) -> Conv2DParams:
        return Conv2DParams(self.pad, self.pad, self.stride, self.stride, 1, 1, self.groups)

    def out_hw(self) -> tuple[int, int]:
        return conv_out_shape(self.h, self.w, self.c, self.r, self.r, self.k, self.params())

    def epilogue(self) -> Epilogue:
        if self.linear:
            return Epilogue.int8()
        if self.relu6:
            return Epilogue.int8(relu6_q=Q6)
        return Epilogue.int8(relu=True)

    def ops_per_image(self) -> int:
        ho, wo = self.out_hw()
        return 2 * ho * wo * self.k * self.r * self.r * (self.c // self.groups)


def resnet50() -> list[LayerSpec]:
    L = [LayerSpec("stem", 224, 224, 3, 64, 7, 2)]
    cin, hw = 64, 56
    for si, (width, blocks) in enumerate([(64, 3), (128, 4), (256, 6), (512, 3)]):
        for b in range(blocks):
            stride = 2 if (b == 0 and si > 0) else 1
            out = width * 4
            L.append(LayerSpec(f"s{si + 1}b{b + 1}.conv1", hw, hw, cin, width, 1, 1))
            L.append(LayerSpec(f"s{si + 1}b{b + 1}.conv2", hw, hw, width, width, 3, stride))
            hw2 = hw // stride
            L.append(LayerSpec(f"s{si + 1}b{b + 1}.conv3", hw2, hw2, width, out, 1, 1))
            if b == 0:
                L.append(LayerSpec(f"s{si + 1}b{b + 1}.proj", hw, hw, cin, out, 1, stride))
            cin, hw = out, hw2
    return L


def mobilenetv2() -> list[LayerSpec]:
    L = [LayerSpec("stem", 224, 224, 3, 32, 3, 2, relu6=True)]
    cin, hw = 32, 112
    for gi, (t, c, n, s) in enumerate([(1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1),
                                       (6, 160, 3, 2), (6, 320, 1, 1)]):
        for b in range(n):
            stride = s if b == 0 else 1
            hid = cin * t
            tag = f"g{gi + 1}b{b + 1}"
            if t != 1:
                L.append(LayerSpec(f"{tag}.expand", hw, hw, cin, hid, 1, 1, relu6=True))
            L.append(LayerSpec(f"{tag}.dw", hw, hw, hid, hid, 3, stride, groups=hid, relu6=True))
            hw = (hw + 2 - 3) // stride + 1
            L.append(LayerSpec(f"{tag}.project", hw, hw, hid, c, 1, 1, linear=True))
            cin = c
    L.append(LayerSpec("final", hw, hw, cin, 1280, 1, 1, relu6=True))
    return L


NETS = {"resnet50": resnet50, "mobilenetv2": mobilenetv2}


class NetData:
    """Device tensors for every layer of a spec list: input, weights, bias, scale, output.
    Tensor ids per layer i: 100*i + {1 input, 2 weights, 3 bias, 4 scale}; `first_layer` numbers the
    first spec as layer `first_layer` of its table (a slice of a table keeps the table's tensors)."""

    def __init__(self, specs: list[LayerSpec], batch: int, seed: int, device, image_offset: int = 0,
                 first_layer: int = 0):
        self.specs, self.batch, self.seed = specs, batch, seed
        act = torch.from_numpy(act_table()).to(device)
        wtab = torch.from_numpy(weight_table()).to(device)
        self.layers = []
        for i, sp in enumerate(specs, start=first_layer):
            x = torch.empty((batch, sp.h, sp.w, sp.c), dtype=torch.int8, device=device)
            synth.fill_s8_table(x, seed + image_offset, 100 * i + 1, act)
            w = synth.fill_s8_table(torch.empty((sp.k, sp.r, sp.r, sp.c // sp.groups), dtype=torch.int8,
                                                device=device), seed, 100 * i + 2, wtab)
            b = synth.fill_i32_uniform(torch.empty(sp.k, dtype=torch.int32, device=device), seed, 100 * i + 3,
                                       -2**15, 2**15)
            s = torch.from_numpy(synth.scales_f32(sp.k, seed, 100 * i + 4)).to(device)
            ho, wo = sp.out_hw()
            y = torch.empty((batch, ho, wo, sp.k), dtype=torch.int8, device=device)
            self.layers.append((sp, x, w, b, s, y))

    def run_layer(self, i: int, stream=None) -> None:
        sp, x, w, b, s, y = self.layers[i]
        conv2d_s8_into(y, x, w, b, s, self.batch, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.params(), sp.epilogue(),
                       stream)

    def run(self, stream=None) -> None:
        for i in range(len(self.layers)):
            self.run_layer(i, stream)


def act_table() -> np.ndarray:
    return synth.quantile_table("halfnormal", 40.0, 0, 127)


def weight_table() -> np.ndarray:
    return synth.quantile_table("normal", 30.0, -127, 127)


def host_layer_tensors(sp: LayerSpec, i: int, seed: int, img0: int, nimg: int):
    """CPU copies (for checking) of images [img0, img0+nimg) of layer i's input and its weights."""
    per = sp.h * sp.w * sp.c
    x = synth.s8_table_host(seed, 100 * i + 1, act_table(), img0 * per, nimg * per).reshape(nimg, sp.h, sp.w, sp.c)
    w = synth.s8_table_host(seed, 100 * i + 2, weight_table(), 0, sp.k * sp.r * sp.r * (sp.c // sp.groups))
    w = w.reshape(sp.k, sp.r, sp.r, sp.c // sp.groups)
    b = synth.i32_uniform_host(seed, 100 * i + 3, -2**15, 2**15, 0, sp.k)
    s = synth.scales_f32(sp.k, seed, 100 * i + 4)
    return x, w, b, s


# ---------------------------------------------------------------------------------------------
# Chained networks: every layer of the table fed by the previous one, with the residual adds fused
# into the conv epilogues, ResNet-50's 3x3/2 max pool after the stem and a global average pool at
# the end.  Weights, biases and scales are the seeded per-layer tensors of NetData (same ids).

RES_SCALE = 0.5  # scale of the shortcut branch in the fused residual add (synthetic network)


@dataclass(frozen=True)
class ChainOp:
    kind: str          # "conv", "maxpool", "avgpool"
    layer: int = -1    # index into the spec list (conv)
    src: int = 0       # input buffer id
    dst: int = 0       # output buffer id
    res: int = -1      # residual buffer id (conv with fused add), -1 = none


def chain_plan(name: str) -> list[ChainOp]:
    """Data flow of the chained network over buffer ids (0 = network input)."""
    specs = NETS[name]()
    ops: list[ChainOp] = []
    nxt = 1
    if name == "resnet50":
        ops.append(ChainOp("conv", 0, 0, nxt)); nxt += 1
        ops.append(ChainOp("maxpool", -1, nxt - 1, nxt)); cur = nxt; nxt += 1
        i = 1
        while i < len(specs):
            conv1, conv2, conv3 = i, i + 1, i + 2
            proj = i + 3 if i + 3 < len(specs) and specs[i + 3].name.endswith(".proj") else -1
            ops.append(ChainOp("conv", conv1, cur, nxt)); b1 = nxt; nxt += 1
            ops.append(ChainOp("conv", conv2, b1, nxt)); b2 = nxt; nxt += 1
            short = cur
            if proj >= 0:
                ops.append(ChainOp("conv", proj, cur, nxt)); short = nxt; nxt += 1
            ops.append(ChainOp("conv", conv3, b2, nxt, res=short)); cur = nxt; nxt += 1
            i += 4 if proj >= 0 else 3
    elif name == "mobilenetv2":
        ops.append(ChainOp("conv", 0, 0, nxt)); cur = nxt; nxt += 1
        i = 1
        while i < len(specs) - 1:
            blk_in = cur
            if specs[i].name.endswith(".expand"):
                ops.append(ChainOp("conv", i, cur, nxt)); cur = nxt; nxt += 1; i += 1
            dw = specs[i]
            ops.append(ChainOp("conv", i, cur, nxt)); cur = nxt; nxt += 1; i += 1
            proj = specs[i]
            cin = specs[i - 1].c if not specs[i - 2].name.endswith(".expand") else specs[i - 2].c
            residual = dw.stride == 1 and proj.k == cin
            ops.append(ChainOp("conv", i, cur, nxt, res=blk_in if residual else -1)); cur = nxt; nxt += 1; i += 1
        ops.append(ChainOp("conv", len(specs) - 1, cur, nxt)); cur = nxt; nxt += 1
    else:
        raise ValueError(name)
    ops.append(ChainOp("avgpool", -1, cur, nxt))
    return ops


class ChainedNet:
    """A whole int8 network on one device.  forward(x) runs every op of chain_plan on the stream;
    intermediate buffers are allocated once per batch size and reused."""

    def __init__(self, name: str, seed: int, device):
        self.name, self.seed, self.device = name, seed, torch.device(device)
        self.specs = NETS[name]()
        self.plan = chain_plan(name)
        wtab = torch.from_numpy(weight_table()).to(self.device)
        self.weights = []
        for i, sp in enumerate(self.specs):
            w = synth.fill_s8_table(torch.empty((sp.k, sp.r, sp.r, sp.c // sp.groups), dtype=torch.int8,
                                                device=self.device), seed, 100 * i + 2, wtab)
            b = synth.fill_i32_uniform(torch.empty(sp.k, dtype=torch.int32, device=self.device), seed, 100 * i + 3,
                                       -2**15, 2**15)
            s = torch.from_numpy(synth.scales_f32(sp.k, seed, 100 * i + 4)).to(self.device)
            self.weights.append((w, b, s))
        self._bufs: dict[int, dict[int, torch.Tensor]] = {}

    def _buffers(self, n: int, x: torch.Tensor) -> dict[int, torch.Tensor]:
        if n not in self._bufs:
            shapes = {0: tuple(x.shape[1:])}
            bufs = {}
            for op in self.plan:
                h, w, c = shapes[op.src]
                if op.kind == "conv":
                    sp = self.specs[op.layer]
                    ho, wo = sp.out_hw()
                    shapes[op.dst] = (ho, wo, sp.k)
                elif op.kind == "maxpool":
                    shapes[op.dst] = ((h + 2 - 3) // 2 + 1, (w + 2 - 3) // 2 + 1, c)
                else:
                    shapes[op.dst] = (1, 1, c)
                bufs[op.dst] = torch.empty((n,) + shapes[op.dst], dtype=torch.int8, device=self.device)
            self._bufs[n] = bufs
        return self._bufs[n]

    def forward(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """x: int8 [n, 224, 224, 3] on the device -> pooled int8 features [n, C_last]."""
        n = x.shape[0]
        bufs = self._buffers(n, x)
        bufs[0] = x
        for op in self.plan:
            src, dst = bufs[op.src], bufs[op.dst]
            if op.kind == "conv":
                sp = self.specs[op.layer]
                w, b, s = self.weights[op.layer]
                if op.res >= 0:
                    conv2d_s8_add_into(dst, src, w, b, s, bufs[op.res], RES_SCALE, n, sp.h, sp.w, sp.c, sp.r, sp.r,
                                       sp.k, sp.params(), sp.epilogue(), stream)
                else:
                    conv2d_s8_into(dst, src, w, b, s, n, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.params(),
                                   sp.epilogue(), stream)
            elif op.kind == "maxpool":
                maxpool_s8(src, 3, 3, 2, 1, out=dst, stream=stream)
            else:
                global_avgpool_s8(src, out=dst.view(n, -1), stream=stream)
        return bufs[self.plan[-1].dst].view(n, -1)
