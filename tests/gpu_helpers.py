"""Shared helpers of the GPU parity tests (device buffers via torch, the C
ABI via lbk, the CPU oracle as the checker)."""

from __future__ import annotations

import numpy as np
import torch

import lbk
import oracle as orc
import synth

DEV = "cuda:0"

_ctx = None


def ctx() -> lbk.Context:
    global _ctx
    if _ctx is None:
        _ctx = lbk.Context(0)
    return _ctx


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).view(np.uint32)


# Element-wise relative error. A combined output row is a sum of terms
# (moe.rs:116-147: c_j * dot_j over the routed experts, then the shared dot;
# plus the residual in a block), and the rounding error of a sum is bounded
# relative to the magnitude of its terms, not to the sum, which can cancel to
# almost nothing. So the error of element i is taken against its term
# magnitude mag_i (moe_term_magnitude) where the test supplies it, else
# against |want_i|; in both cases with a floor of REL_FLOOR times the largest
# denominator, so that an element a thousand times below the row's largest is
# held to an absolute error of 1e-8 of that largest magnitude instead of to its own size.
REL_FLOOR = 1e-3


def norm_err(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / max |want| (norm-wise relative error)."""
    scale = float(np.max(np.abs(want))) or 1.0
    return float(np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)))) / scale


def rel_err(got: np.ndarray, want: np.ndarray, mag: np.ndarray | None = None, floor: float = REL_FLOOR) -> float:
    """Element-wise relative error: max_i |got_i - want_i| / max(d_i, floor * max d),
    d = mag (term magnitudes) if given, else |want|."""
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    d = np.abs(w) if mag is None else np.asarray(mag, np.float64).reshape(w.shape)
    scale = float(np.max(d)) or 1.0
    return float(np.max(np.abs(g - w) / np.maximum(d, floor * scale)))


def errs(got: np.ndarray, want: np.ndarray, mag: np.ndarray | None = None) -> str:
    kind = "of term magnitudes" if mag is not None else "of |want|"
    return (f"element-wise {rel_err(got, want, mag):.3e} ({kind}, floor {REL_FLOOR}), "
            f"norm-wise {norm_err(got, want):.3e}")


def moe_term_magnitude(table, ids, coefs, x) -> np.ndarray:
    """Per output row of one token's MoE step: |shared dot| + sum_j |c_j| |routed dot_j|,
    the magnitudes the reference's combine adds, from the oracle (one expert at a time)."""
    x = np.ascontiguousarray(x, np.float32)
    shared = orc.moe_routed(table, np.asarray(ids[:1], np.uint32), np.zeros(1, np.float32), x).astype(np.float64)
    mag = np.abs(shared)
    for e, c in zip(ids, coefs):
        dot = orc.moe_routed(table, np.array([e], np.uint32), np.ones(1, np.float32), x).astype(np.float64) - shared
        mag += abs(float(c)) * np.abs(dot)
    return mag


def planar_dev(ty: int, gguf: np.ndarray, in_w: int) -> torch.Tensor:
    return dev(synth.planar_np(ty, gguf, in_w))


def matrix(ty, in_w, out_w, t: torch.Tensor, layout=lbk.LAYOUT_GGUF) -> lbk.Matrix:
    return lbk.matrix(ty, in_w, out_w, t, layout)


def expect_status(code: int) -> lbk.ErrorDetail:
    st = ctx().sync_status()
    assert st == code, f"status {st} ({lbk.STATUS.get(st)}), expected {code}"
    return ctx().last_detail


def clean_status() -> None:
    st = ctx().sync_status()
    assert st == 0, f"unexpected device status {st} ({lbk.STATUS.get(st)}): {ctx().last_detail.index}"


def make_layer_np(rng, H, F, E, gty=orc.TYPE_IQ2_S, dty=orc.TYPE_IQ3_S, sty=orc.TYPE_Q4_K, sdty=orc.TYPE_Q4_K):
    """Host expert table in the order of the synthetic generator: router,
    experts 0..E-1 (gate, up, down), shared (gate, up, down)."""
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    experts = []
    for _ in range(E):
        g = synth.packed_np(rng, gty, H, F)
        u = synth.packed_np(rng, gty, H, F)
        d = synth.packed_np(rng, dty, F, H)
        experts.append((gty, g, gty, u, dty, d, H, F))
    sg = synth.packed_np(rng, sty, H, F)
    su = synth.packed_np(rng, sty, H, F)
    sd = synth.packed_np(rng, sdty, F, H)
    shared = (sty, sg, sty, su, sdty, sd, H, F)
    return router, experts, shared


def upload_layer(router, experts, shared, layout, top_k, weight_scale=2.826, bias=None):
    """Device copies + an lbk.MoeLayer; returns (layer, keepalive)."""
    H = shared[6]
    E = len(experts)
    keep = []

    def up(ty, b, in_w):
        t = planar_dev(ty, b, in_w) if layout == lbk.LAYOUT_PLANAR else dev(b)
        keep.append(t)
        return t

    def ex(e):
        gty, gb, uty, ub, dty, db, h, f = e
        return lbk.Expert(
            matrix(gty, h, f, up(gty, gb, h), layout),
            matrix(uty, h, f, up(uty, ub, h), layout),
            matrix(dty, f, h, up(dty, db, f), layout),
        )

    dex = [ex(e) for e in experts]
    sh = ex(shared)
    rt = dev(router)
    keep.append(rt)
    rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, H, E, rt.data_ptr(), rt.numel() * 4)
    b = dev(np.zeros(E, np.float32) if bias is None else bias)
    keep.append(b)
    layer = lbk.MoeLayer(ctx(), dex, sh, rm, b, top_k, weight_scale)
    return layer, keep


def topk_margins(router: np.ndarray, xs: np.ndarray, bias: np.ndarray, k: int) -> np.ndarray:
    """Per token: the gap between the k-th and (k+1)-th selection score
    (sigmoid(logit) + bias, route_experts_into's sort key). Top-k identity on a
    test input is only meaningful where this gap is well above rounding."""
    out = []
    for x in xs:
        logits = orc.gemv_f32(router.shape[1], router.shape[0], router.reshape(-1), x).astype(np.float64)
        s = np.sort(1.0 / (1.0 + np.exp(-logits)) + bias.astype(np.float64))[::-1]
        out.append(s[k - 1] - s[k])
    return np.array(out)
