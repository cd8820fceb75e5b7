"""One encoder layer on the device (libpktito_b200.encoder.layer_dev), the
batch's segments at once, against the oracle's composition of the same
steps a segment at a time (layer(), core/encoder.c:338-368): normq, the
products, siluq_tile, the position embeddings quantized once, att_item,
the quantization of its output, glu_item + dw_item, and the out norm, each
step restated in oracle/q8_oracle.c and pinned to the reference's own.

The model's shapes (d_model 1024, ff 4096, 8 heads, kernel 9) with seeded
weights; segments of 1, 7 and 20 frames (a segment shorter than the
convolution's taps, one under a block of queries); blocks of 32 and of 64
(the reference's fast mode).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

D, F, H, K, EPS = 1024, 4096, 8, 9, 1e-5


def seeded_layer(seed: int) -> dict:
    """The layer's weights on the host: PK_Q8 bytes and row scales a
    product, the norms, the position biases and the convolution's taps."""
    from libpktito_b200.encoder import PRODUCTS, product_shapes
    g = np.random.default_rng(seed)
    L = {}
    for name in PRODUCTS:
        rows, n = product_shapes(D, F)[name]
        L[name] = (O.pack_q8(g.integers(-127, 128, (rows, n), dtype=np.int8)),
                   (1e-4 + 9e-4 * g.random(rows)).astype(np.float32))
    for name in ("ff1", "att", "conv", "ff2", "out"):
        L[name + "_nw"] = (1 + 0.1 * g.standard_normal(D)).astype(np.float32)
        L[name + "_nb"] = (0.1 * g.standard_normal(D)).astype(np.float32)
    L["bias_u"], L["bias_v"] = ((0.1 * g.standard_normal(D)).astype(np.float32) for _ in range(2))
    L["dw"] = (0.3 * g.standard_normal(D * K)).astype(np.float32)
    L["dw_b"] = (0.1 * g.standard_normal(D)).astype(np.float32)
    return L


def device_layer(pkb, L: dict) -> dict:
    import torch
    out = {}
    for k, v in L.items():
        if isinstance(v, tuple):
            from libpktito_b200.encoder import product_shapes
            rows, n = product_shapes(D, F)[k]
            src = torch.from_numpy(v[0]).cuda()
            w = torch.empty(rows * n, dtype=torch.int8, device="cuda")
            pkb.repack_q8_dev(w, src, rows, n)
            out[k] = (w, torch.from_numpy(v[1]).cuda())
        else:
            out[k] = torch.from_numpy(v).cuda()
    return out


def oracle_layer(x: np.ndarray, T: int, L: dict, ape: np.ndarray, qb: int, rmode: int) -> np.ndarray:
    """layer() on one segment, step by step with the oracle (x: T rows of D)."""
    x = x.copy()

    def prod(out, name, q, d, n, add, Tn):
        w, ws = L[name]
        rows = ws.size
        O.gemm_q8(out, rows, w, ws, None, rows, q, d, n, qb, Tn, add, rmode)

    def ff(pre):
        q, d = O.layernorm_quantize(x, D, T, D, qb, L[pre + "_nw"], L[pre + "_nb"], EPS, rmode)
        u = np.zeros(T * F, np.float32)
        prod(u, pre + "_up", q, d, D, False, T)
        q2, d2 = O.silu_quantize(u, F, T, F, qb, rmode)
        prod(x, pre + "_down", q2, d2, F, True, T)

    ff("ff1")
    q, d = O.layernorm_quantize(x, D, T, D, qb, L["att_nw"], L["att_nb"], EPS, rmode)
    Q, Kr, V = (np.zeros(T * D, np.float32) for _ in range(3))
    for name, out in (("q", Q), ("k", Kr), ("v", V)):
        prod(out, name, q, d, D, False, T)
    R = 2 * T - 1
    aq, ad = O.quantize(ape, D, qb, R, D, rmode)
    Pr = np.zeros(R * D, np.float32)
    prod(Pr, "pos", aq, ad, D, False, R)
    dk = D // H
    Tp, Pp = (T + 15) // 16 * 16, (R + 15) // 16 * 16 + 16
    vp = np.ascontiguousarray(V.reshape(T, D // 16, 16).transpose(1, 0, 2)).reshape(-1)
    o = O.attention(Q, D, O.panels_kp(Kr, T, Tp, D, dk), O.panels_kp(Pr, R, Pp, D, dk), vp, L["bias_u"],
                    L["bias_v"], T, D, H, rmode)
    qo, do = O.quantize(o, D, qb, T, D, rmode)
    prod(x, "o", qo, do, D, True, T)
    q, d = O.layernorm_quantize(x, D, T, D, qb, L["conv_nw"], L["conv_nb"], EPS, rmode)
    U = np.zeros(T * 2 * D, np.float32)
    prod(U, "pw1", q, d, D, False, T)
    qc, dc, _ = O.dwconv_quantize(U, 2 * D, T, D, L["dw"], L["dw_b"], K, True, qb, rmode)
    prod(x, "pw2", qc, dc, D, True, T)
    ff("ff2")
    return O.layernorm(x, D, T, D, L["out_nw"], L["out_nb"], EPS, rmode).reshape(-1)


@pytest.mark.parametrize("qb,rmode", [(32, O.RN), (64, O.RN), (32, O.RZ)])
def test_layer_on_the_device_is_the_references(pkb, cuda_device, qb, rmode):
    import torch
    from libpktito_b200.encoder import Batch, Buffers, layer_dev
    L = seeded_layer(5)
    Ld = device_layer(pkb, L)
    Ts = [20, 1, 7]
    segs, f, r = [], 0, 0
    for T in Ts:
        segs.append((T, f, r))
        f += T
        r += 2 * T - 1
    batch = Batch(segs)
    g = np.random.default_rng(6)
    x = g.standard_normal(batch.frames * D).astype(np.float32)
    ape = g.standard_normal(batch.positions * D).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    aq = torch.empty(batch.positions * D, dtype=torch.int8, device="cuda")
    ad = torch.empty(batch.positions * D // qb, device="cuda")
    pkb.quantize_dev(aq, ad, torch.from_numpy(ape).cuda(), D, batch.positions, D, qb, rmode)
    buf = Buffers(torch, batch.frames, batch.positions, D, F, qb)
    layer_dev(xd, Ld, batch, aq, ad, D, F, H, K, qb, EPS, buf, rmode)
    torch.cuda.synchronize()
    got = xd.cpu().numpy().reshape(batch.frames, D)
    for T, f, r in segs:
        want = oracle_layer(x[f * D:(f + T) * D], T, L, ape[r * D:(r + 2 * T - 1) * D], qb, rmode)
        assert got[f:f + T].reshape(-1).tobytes() == want.tobytes(), (T, qb, rmode)
