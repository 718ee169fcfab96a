"""A sequence of int8 NHWC conv layers run through the C ABI, with a copy/compute pipeline for
host-resident batches.

``ConvStack.forward`` runs the layers on device tensors (activations stay int8 in HBM between
layers; intermediate buffers are allocated once per batch size and reused).

``ConvStack.run_host`` takes pinned host input / output buffers and overlaps the transfers with
the kernels: the batch is cut into chunks of images (images are independent), and three CUDA
streams carry host->device copies of chunk i+1, the layers of chunk i and device->host copies of
chunk i-1 at the same time.  Each slot of device buffers is reused only after the events of the
chunk that last used it have completed.  The streams and slot buffers are created on the first
call and reused by later calls with the same chunk shape.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .conv import Conv2DParams, Epilogue, conv2d_s8_into, conv_out_shape


@dataclass
class ConvLayer:
    w: torch.Tensor                 # int8 [k, r, s, c / groups]
    bias: torch.Tensor | None       # int32 [k]
    scale: torch.Tensor | None      # fp32 [k]
    params: Conv2DParams
    epi: Epilogue


class ConvStack:
    def __init__(self, layers: list[ConvLayer], in_hwc: tuple[int, int, int]):
        self.layers = layers
        self.shapes = [tuple(in_hwc)]
        h, w, c = in_hwc
        for L in layers:
            k, r, s, _ = L.w.shape
            ho, wo = conv_out_shape(h, w, c, r, s, k, L.params)
            h, w, c = ho, wo, k
            self.shapes.append((h, w, c))
        self.out_dtype = layers[-1].epi.torch_dtype
        self._bufs: dict[tuple[int, int], list[torch.Tensor]] = {}
        # run_host's side streams and input slots, created once per (device, chunk shape, slots)
        self._pipes: dict[tuple, tuple[list[torch.cuda.Stream], list[torch.Tensor]]] = {}

    def _pipeline(self, device, chunk: int, slots: int, x_shape: tuple, x_dtype):
        key = (device, chunk, slots, x_shape, x_dtype)
        if key not in self._pipes:
            streams = [torch.cuda.Stream(device) for _ in range(3)]
            x_slots = [torch.empty((chunk,) + x_shape, dtype=x_dtype, device=device) for _ in range(slots)]
            self._pipes[key] = (streams, x_slots)
        return self._pipes[key]

    def _buffers(self, n: int, slot: int, device) -> list[torch.Tensor]:
        key = (n, slot)
        if key not in self._bufs:
            bufs = []
            for i, L in enumerate(self.layers):
                h, w, c = self.shapes[i + 1]
                bufs.append(torch.empty((n, h, w, c), dtype=L.epi.torch_dtype, device=device))
            self._bufs[key] = bufs
        return self._bufs[key]

    def forward(self, x: torch.Tensor, slot: int = 0, stream=None) -> torch.Tensor:
        """x: int8 [n, h, w, c] on the device.  Returns the last layer's output (a reused buffer)."""
        n = x.shape[0]
        bufs = self._buffers(n, slot, x.device)
        cur = x
        for i, L in enumerate(self.layers):
            h, w, c = self.shapes[i]
            k, r, s, _ = L.w.shape
            conv2d_s8_into(bufs[i], cur, L.w, L.bias, L.scale, n, h, w, c, r, s, k, L.params, L.epi, stream)
            cur = bufs[i]
        return cur

    def run_host(self, h_x: torch.Tensor, h_y: torch.Tensor, chunk: int = 64, slots: int = 3,
                 device=None) -> None:
        """Pipelined host-to-host pass: h_x pinned int8 [n,h,w,c] -> h_y pinned [n, ho, wo, k].

        Enqueued asynchronously on three side streams that join the current stream at the end;
        the caller synchronizes (or records an event on the current stream)."""
        device = device or torch.device("cuda", torch.cuda.current_device())
        n = h_x.shape[0]
        cur = torch.cuda.current_stream(device)
        (s_in, s_cmp, s_out), x_slots = self._pipeline(device, chunk, slots, tuple(h_x.shape[1:]), h_x.dtype)
        # every side stream starts after all work already on the current stream, which includes the
        # previous call's joins: the reused slots are free again
        start = torch.cuda.Event()
        start.record(cur)
        for s in (s_in, s_cmp, s_out):
            s.wait_event(start)
        in_done, cmp_done, out_done = {}, {}, {}
        nchunks = (n + chunk - 1) // chunk
        for i in range(nchunks):
            b0, b1 = i * chunk, min(n, (i + 1) * chunk)
            m = b1 - b0
            slot = i % slots
            xs = x_slots[slot][:m]
            with torch.cuda.stream(s_in):
                if i >= slots:
                    s_in.wait_event(cmp_done[i - slots])  # x slot consumed by its last chunk
                xs.copy_(h_x[b0:b1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                in_done[i] = ev
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(in_done[i])
                if i >= slots:
                    s_cmp.wait_event(out_done[i - slots])  # y slot copied out
                y = self.forward(xs, slot=slot, stream=s_cmp)
                ev = torch.cuda.Event()
                ev.record(s_cmp)
                cmp_done[i] = ev
            with torch.cuda.stream(s_out):
                s_out.wait_event(cmp_done[i])
                h_y[b0:b1].copy_(y, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_out)
                out_done[i] = ev
        for s in (s_in, s_cmp, s_out):
            cur.wait_stream(s)
