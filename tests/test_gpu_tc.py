"""GPU parity: grouped row dots of IQ2_S and IQ3_S matrices on the tcgen05
tensor cores (lbk_tc_grouped_dots, int8 MMA with one accumulator per scale
group: 16 weights for IQ2_S, 32 for IQ3_S) against the CPU oracle's gemv per
token, bit for bit: matrices of K = 1536 to 4096, row counts that are not multiples of the 128-row tile,
groups of 1 to 32 tokens (both MMA widths, N = 16 and 32), tokens repeated
across groups, and a malformed job reported without any write.
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
import synth
from gpu_helpers import bits, clean_status, ctx, dev, expect_status, host, planar_dev

pytestmark = pytest.mark.gpu

Q8I = 304  # internal Q8_K image bytes per 256 block


def q8_image(x: np.ndarray) -> np.ndarray:
    """The kernels' token image of Q8_K(x): per block qs, bsums, d, padding."""
    ref = orc.quantize_q8k(x).reshape(-1, orc.Q8K_BLOCK_BYTES)
    img = np.zeros((ref.shape[0], Q8I), dtype=np.uint8)
    img[:, :256] = ref[:, 4:260]
    img[:, 256:288] = ref[:, 260:292]
    img[:, 288:292] = ref[:, 0:4]
    return img.reshape(-1)


def jobs_for(groups, rows_of):
    """One job per (matrix, 128-row tile, run of <= 32 pairs of its group)."""
    jobs, pair_tokens = [], []
    for m, toks in groups:
        p0 = len(pair_tokens)
        pair_tokens += list(toks)
        for c in range(0, len(toks), 32):
            for r0 in range(0, rows_of[m], 128):
                jobs.append((m, r0, p0 + c, min(32, len(toks) - c)))
    return np.array(jobs, dtype=np.int32).reshape(-1, 4), np.array(pair_tokens, dtype=np.int32)


@pytest.mark.parametrize("ty,k", [(orc.TYPE_IQ2_S, 2048), (orc.TYPE_IQ2_S, 4096), (orc.TYPE_IQ3_S, 1536),
                                  (orc.TYPE_IQ3_S, 4096)])
def test_tc_grouped_dots_match_oracle_gemv(ty, k):
    rng = np.random.default_rng(17 + k + ty)
    shapes = [200, 128, 384, 77]
    ws = [synth.packed_np(rng, ty, k, rows) for rows in shapes]
    wd = [planar_dev(ty, w, k) for w in ws]
    T = 40
    xs = rng.standard_normal((T, k)).astype(np.float32)
    q8 = dev(np.concatenate([q8_image(x) for x in xs]))
    groups = [(0, [3]), (1, list(range(32))), (2, list(rng.integers(0, T, 17))), (3, list(range(5, 40))),
              (0, [1, 1, 2])]
    jobs, pair_tokens = jobs_for(groups, shapes)
    stride = max(shapes)
    mats = dev(lbk.tc_matrices([(t.data_ptr(), rows, k // 256, 0) for t, rows in zip(wd, shapes)]))
    dots = torch.full((len(pair_tokens), stride), float("nan"), device="cuda")
    ctx().tc_grouped_dots(mats, len(shapes), dev(jobs), len(jobs), q8, k // 256 * Q8I, dev(pair_tokens), dots, stride,
                          type=ty)
    clean_status()
    got = host(dots)
    want = {}
    p = 0
    for m, toks in groups:
        for t in toks:
            key = (m, int(t))
            if key not in want:
                want[key] = orc.gemv(ty, k, shapes[m], ws[m], xs[t])[0]
            np.testing.assert_array_equal(bits(got[p, :shapes[m]]), bits(want[key]), err_msg=f"pair {p}: matrix {m} token {t}")
            p += 1


def test_tc_grouped_dots_reject_malformed_job():
    rng = np.random.default_rng(5)
    k, rows = 2048, 128
    w = planar_dev(orc.TYPE_IQ2_S, synth.packed_np(rng, orc.TYPE_IQ2_S, k, rows), k)
    q8 = dev(q8_image(rng.standard_normal(k).astype(np.float32)))
    mats = dev(lbk.tc_matrices([(w.data_ptr(), rows, k // 256, 0)]))
    dots = torch.full((1, rows), float("nan"), device="cuda")
    bad = np.array([[0, 0, 0, 33]], dtype=np.int32)  # more pairs than a job holds
    ctx().tc_grouped_dots(mats, 1, dev(bad), 1, q8, k // 256 * Q8I, dev(np.zeros(1, np.int32)), dots, rows)
    d = expect_status(15)  # LBK_INVALID_PARAMETER
    assert d.index == 0
    assert np.isnan(host(dots)).all()
