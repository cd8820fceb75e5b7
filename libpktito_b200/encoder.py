"""One FastConformer encoder layer on the device, for a batch of segments.

The reference runs `layer()` (core/encoder.c:338-368) one segment at a time
on the host, its int8 products through the backend table and its float steps
between them in core/encoder.c. Here the same layer runs on the GPU over a
batch of segments whose frames lie one after another (row t of the batch is
frame t - f_s of segment s), every step a kernel of this library on device
rows, so that nothing crosses PCIe between the layer's input and its output:

    ff(ff1)           normq -> FF-up -> siluq_tile -> FF-down (added)     :342, ff() :329-336
    attention         normq -> q rows, K, V, P rows (P from the position
                      embeddings quantized once a forward pass) -> att_item
                      over every segment and head -> quantize o -> o (added)  :344-355
    convolution       normq -> pw1 -> glu_item + dw_item -> pw2 (added)    :357-363
    ff(ff2)                                                              :365
    norm              k_layernorm in place                                 :367

Each step is the reference's operation for operation (the kernels' own
docstrings say how); the products' columns are independent and the
attention and the depthwise convolution are taken a segment at a time, so
each segment's frames come out as the reference's `layer()` makes them for
that segment alone (tests/test_gpu_encoder.py holds them to the oracle's
composition of the same steps).

Weights are device tensors: int8 matrices as `repack_q8_dev` rows (from the
model file's PK_Q8 panels) with their row scales.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import (RN, attention_rows_dev, dwconv_quantize_dev, gemm_q8_dev, layernorm_dev, layernorm_quantize_dev,
               quantize_dev, silu_quantize_dev)

# the products of a layer, (name, rows, inputs) with D the model's width and F
# its feed-forward width (core/model.h:45-55)
PRODUCTS = ("ff1_up", "ff1_down", "q", "k", "v", "pos", "o", "pw1", "pw2", "ff2_up", "ff2_down")


def product_shapes(D: int, F: int) -> dict:
    return {"ff1_up": (F, D), "ff1_down": (D, F), "q": (D, D), "k": (D, D), "v": (D, D), "pos": (D, D),
            "o": (D, D), "pw1": (2 * D, D), "pw2": (D, D), "ff2_up": (F, D), "ff2_down": (D, F)}


@dataclass
class Batch:
    """A batch of segments: frames of segment s at rows f_s .. f_s + T_s - 1,
    its 2 T_s - 1 position rows at p_s .. of the position embeddings."""
    segs: list  # (T, f, p)

    @property
    def frames(self) -> int:
        return sum(t for t, _, _ in self.segs)

    @property
    def positions(self) -> int:
        return sum(2 * t - 1 for t, _, _ in self.segs)


class Buffers:
    """The layer's device scratch for a batch of M frames and R position rows."""

    def __init__(self, torch, M: int, R: int, D: int, F: int, qb: int):
        dev = "cuda"
        self.act_q = torch.empty(M * max(D, F), dtype=torch.int8, device=dev)
        self.act_d = torch.empty(M * max(D, F) // qb, device=dev)
        self.u = torch.empty(M * max(F, 2 * D), device=dev)
        self.q = torch.empty(M * D, device=dev)
        self.k = torch.empty(M * D, device=dev)
        self.v = torch.empty(M * D, device=dev)
        self.p = torch.empty(max(R, 1) * D, device=dev)
        self.o = torch.empty(M * D, device=dev)


def _ff(x, L: dict, pre: str, M: int, D: int, F: int, qb: int, eps: float, buf: Buffers, rmode: int, s) -> None:
    """ff() (core/encoder.c:329-336): x += down(siluq(up(normq(x))))"""
    layernorm_quantize_dev(buf.act_q, buf.act_d, x, D, M, D, qb, L[pre + "_nw"], L[pre + "_nb"], eps, rmode, s)
    up, ups = L[pre + "_up"]
    gemm_q8_dev(buf.u, F, up, ups, None, F, buf.act_q, buf.act_d, D, qb, M, False, rmode, s)
    silu_quantize_dev(buf.act_q, buf.act_d, buf.u, F, M, F, qb, rmode, s)
    down, downs = L[pre + "_down"]
    gemm_q8_dev(x, D, down, downs, None, D, buf.act_q, buf.act_d, F, qb, M, True, rmode, s)


def layer_dev(x, L: dict, batch: Batch, ape_q, ape_d, D: int, F: int, H: int, K: int, qb: int, eps: float,
              buf: Buffers, rmode: int = RN, stream=None) -> None:
    """layer() (core/encoder.c:338-368) in place on x, the batch's rows of D
    floats. L: the layer's weights on the device (PRODUCTS as (rows, scales)
    pairs; the norms' w and b as "<name>_nw", "<name>_nb"; bias_u, bias_v;
    the depthwise convolution's taps "dw" [D][K] and bias "dw_b"). ape_q,
    ape_d: the position embeddings of every segment's 2T - 1 positions,
    quantized once a forward pass (core/encoder.c:469)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    M = batch.frames
    _ff(x, L, "ff1", M, D, F, qb, eps, buf, rmode, s)

    # the attention block: q, k and v read one quantized input, the
    # position product the embeddings; att_item over every segment and head
    layernorm_quantize_dev(buf.act_q, buf.act_d, x, D, M, D, qb, L["att_nw"], L["att_nb"], eps, rmode, s)
    for name, out in (("q", buf.q), ("k", buf.k), ("v", buf.v)):
        w, ws = L[name]
        gemm_q8_dev(out, D, w, ws, None, D, buf.act_q, buf.act_d, D, qb, M, False, rmode, s)
    w, ws = L["pos"]
    gemm_q8_dev(buf.p, D, w, ws, None, D, ape_q, ape_d, D, qb, batch.positions, False, rmode, s)
    attention_rows_dev(buf.o, D, buf.q, D, buf.k, D, buf.v, D, buf.p, D, L["bias_u"], L["bias_v"], D, H,
                       batch.segs, rmode, s)
    quantize_dev(buf.act_q, buf.act_d, buf.o, D, M, D, qb, rmode, s)
    w, ws = L["o"]
    gemm_q8_dev(x, D, w, ws, None, D, buf.act_q, buf.act_d, D, qb, M, True, rmode, s)

    # the convolution block: pw1, then GLU + the depthwise convolution
    # (a segment at a time: its taps must not reach across segments) + SiLU,
    # quantized, then pw2
    layernorm_quantize_dev(buf.act_q, buf.act_d, x, D, M, D, qb, L["conv_nw"], L["conv_nb"], eps, rmode, s)
    w, ws = L["pw1"]
    gemm_q8_dev(buf.u, 2 * D, w, ws, None, 2 * D, buf.act_q, buf.act_d, D, qb, M, False, rmode, s)
    for T, f, _ in batch.segs:
        if T:
            u = buf.u[f * 2 * D:]
            qa, da = buf.act_q[f * D:], buf.act_d[f * (D // qb):]
            dwconv_quantize_dev(qa, da, None, D, u, 2 * D, T, D, L["dw"], L["dw_b"], K, True, qb, rmode, s)
    w, ws = L["pw2"]
    gemm_q8_dev(x, D, w, ws, None, D, buf.act_q, buf.act_d, D, qb, M, True, rmode, s)

    _ff(x, L, "ff2", M, D, F, qb, eps, buf, rmode, s)
    layernorm_dev(x, D, x, D, M, D, L["out_nw"], L["out_nb"], eps, rmode, s)
