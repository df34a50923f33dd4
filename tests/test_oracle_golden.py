"""Pins the CPU oracle to the reference's own golden vectors.

Mirrors crates/bridge-quant-layout/tests/oracle_vectors.rs:24-182 (decode,
Q8_K quantize and dot fixtures, bit-exact), src/tables.rs:1581-1593 (codebook
SHA-256 locks), src/q8_k.rs:737-751 (nearest_int ties) and tests/abi.rs:277-300
(exact binary16 conversion).
"""

import hashlib

import numpy as np
import oracle as orc
import pytest
from conftest import REPO, read_golden

TYPES = [
    ("q4-k", orc.TYPE_Q4_K, 144),
    ("q5-k", orc.TYPE_Q5_K, 176),
    ("iq2-s", orc.TYPE_IQ2_S, 82),
    ("iq3-s", orc.TYPE_IQ3_S, 110),
]


def test_golden_manifest_hashes():
    for line in (REPO / "tests/golden/MANIFEST.sha256").read_text().splitlines():
        digest, name = line.split()
        assert hashlib.sha256(read_golden(name)).hexdigest() == digest, name


def test_table_sha256_locks():
    # tables.rs:12, :1043, :1562
    assert hashlib.sha256(orc.table_bytes(0)).hexdigest() == "5ac9831b2e30eb285ef34f8501620f878432d5c04331ad1ae47f977a83ba41a5"
    assert hashlib.sha256(orc.table_bytes(1)).hexdigest() == "e1aa1473412b0552c2174c30ef22ab4073f6a181b85a17056e8249bd2932fd88"
    assert hashlib.sha256(orc.table_bytes(2)).hexdigest() == "bd1af4945a1717c65610b0284e4628b9a1ba3b306fae3a06f6e5f597356e349f"


@pytest.mark.parametrize("name,ty,bb", TYPES)
def test_decode_fixture_bit_exact_row_and_blocks(name, ty, bb):
    enc = np.frombuffer(read_golden(f"decode-{name}.input.bin"), dtype=np.uint8)
    want = np.frombuffer(read_golden(f"decode-{name}.output-f32le.bin"), dtype="<u4")
    row = orc.decode_row(ty, enc, 768)
    np.testing.assert_array_equal(row.view(np.uint32), want)
    for b in range(3):
        blk = orc.decode_row(ty, enc[b * bb : (b + 1) * bb].copy(), 256)
        np.testing.assert_array_equal(blk.view(np.uint32), want[b * 256 : (b + 1) * 256])


def test_decode_f32_fixture_preserves_bits():
    enc = np.frombuffer(read_golden("decode-f32.input.bin"), dtype=np.uint8)
    want = np.frombuffer(read_golden("decode-f32.output-f32le.bin"), dtype="<u4")
    out = orc.decode_row(orc.TYPE_F32, enc, 16)
    np.testing.assert_array_equal(out.view(np.uint32), want)


def test_q8k_fixture_byte_exact():
    x = np.frombuffer(read_golden("q8-k-activations.input-f32le.bin"), dtype="<f4")
    want = np.frombuffer(read_golden("q8-k-activations.output-q8-k.bin"), dtype=np.uint8)
    np.testing.assert_array_equal(orc.quantize_q8k(x), want)


@pytest.mark.parametrize("simd", [False, True])
@pytest.mark.parametrize("name,ty,bb", TYPES)
def test_dot_fixture_bit_exact(name, ty, bb, simd):
    enc = np.frombuffer(read_golden(f"decode-{name}.input.bin"), dtype=np.uint8)
    q8 = np.frombuffer(read_golden("q8-k-activations.output-q8-k.bin"), dtype=np.uint8)
    want = np.frombuffer(read_golden(f"dot-{name}-q8-k.output-f32le.bin"), dtype="<u4")[0]
    got = orc.vec_dot(ty, enc, q8, 768, simd=simd)
    assert np.float32(got).view(np.uint32) == want


def test_nearest_int_ties_to_even():
    # q8_k.rs:737-751
    for v, want in [(-2.5, -2), (-1.5, -2), (-0.5, 0), (0.5, 0), (1.5, 2), (2.5, 2), (3.5, 4)]:
        assert orc.lib().orc_nearest_int(v) == want


def test_binary16_conversion_exact():
    # abi.rs:277-300
    cases = [
        (0x0000, 0x00000000), (0x8000, 0x80000000), (0x0001, 0x33800000), (0x03FF, 0x387FC000),
        (0x0400, 0x38800000), (0x3C00, 0x3F800000), (0xBC00, 0xBF800000), (0x7BFF, 0x477FE000),
    ]
    for h, bits in cases:
        assert np.float32(orc.lib().orc_f16_to_f32(h)).view(np.uint32) == bits
    # every finite half round-trips through numpy's exact conversion
    hs = np.arange(0, 1 << 16, dtype=np.uint16)
    finite = ((hs >> 10) & 0x1F) != 0x1F
    conv = np.array([orc.lib().orc_f16_to_f32(int(h)) for h in hs[finite][::97]], dtype=np.float32)
    np.testing.assert_array_equal(conv, hs[finite][::97].view(np.float16).astype(np.float32))


def test_q8k_zero_blocks_and_rejections():
    # tests/q8_k.rs:11-94
    out = np.full(584, 0xA5, dtype=np.uint8)
    assert orc.quantize_q8k_status(np.zeros(512, np.float32), out) == 0
    assert (out == 0).all()
    sentinel = (np.arange(292) * 37 + 11).astype(np.uint8)
    buf = sentinel.copy()
    assert orc.quantize_q8k_status(np.zeros(0, np.float32), buf) == 2  # ZeroLogicalElements
    assert orc.quantize_q8k_status(np.zeros(255, np.float32), buf) == 3
    assert orc.quantize_q8k_status(np.zeros(256, np.float32), buf[:291].copy()) == 5
    np.testing.assert_array_equal(buf, sentinel)
    for idx in [0, 127, 255, 256, 511]:
        for bad in [np.inf, -np.inf, np.float32(np.nan)]:
            x = np.zeros(512, np.float32)
            x[idx] = bad
            o = np.tile(sentinel, 2)
            before = o.copy()
            assert orc.quantize_q8k_status(x, o) == 8  # NonFiniteActivation
            assert orc.last_detail().index == idx
            np.testing.assert_array_equal(o, before)


def test_scalar_and_simd_dots_agree_on_random_rows():
    rng = np.random.default_rng(5)
    for ty, bb in [(orc.TYPE_Q4_K, 144), (orc.TYPE_Q5_K, 176), (orc.TYPE_IQ2_S, 82), (orc.TYPE_IQ3_S, 110)]:
        w = rng.integers(0, 256, size=16 * bb, dtype=np.uint8)
        for b in range(16):  # finite scales
            w[b * bb : b * bb + 2] = np.frombuffer(np.float16(rng.uniform(0.001, 0.02)).tobytes(), np.uint8)
            if ty in (orc.TYPE_Q4_K, orc.TYPE_Q5_K):
                w[b * bb + 2 : b * bb + 4] = np.frombuffer(np.float16(rng.uniform(0.001, 0.02)).tobytes(), np.uint8)
        q8 = orc.quantize_q8k(rng.standard_normal(4096).astype(np.float32))
        a = orc.vec_dot(ty, w, q8, 4096, simd=False)
        b = orc.vec_dot(ty, w, q8, 4096, simd=True)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_routing_semantics():
    # bridge-model-hy3/tests/routing.rs:46-122
    ids, coefs = orc.route_experts(np.zeros(4, np.float32), np.zeros(4, np.float32), 3, 2.826)
    assert list(ids) == [0, 1, 2]
    assert np.allclose(coefs, 2.826 / 3, atol=1e-6)
    ids, coefs = orc.route_experts(np.array([3, 1, -1, -3], np.float32), np.array([0, 0, 2, 4], np.float32), 2, 2.0)
    assert list(ids) == [2, 3]
    w2 = np.float32(1) / (np.float32(1) + np.exp(np.float32(1)))
    w3 = np.float32(1) / (np.float32(1) + np.exp(np.float32(3)))
    assert abs(coefs[0] - w2 / (w2 + w3) * 2) <= 1e-6
    ids, _ = orc.route_experts(np.array([0, 4, -4, 2], np.float32), np.zeros(4, np.float32), 3, 1.0)
    assert list(ids) == [0, 1, 3]
    fmin = np.finfo(np.float32).min
    ids, coefs = orc.route_experts(np.array([fmin, fmin], np.float32), np.zeros(2, np.float32), 2, 2.826)
    assert (coefs == 0).all()
    assert orc.route_experts_status(np.zeros(3, np.float32), np.zeros(3, np.float32), 0, 1.0) == 16
    assert orc.route_experts_status(np.zeros(3, np.float32), np.zeros(3, np.float32), 4, 1.0) == 16
    assert orc.route_experts_status(np.array([0, np.nan, 0], np.float32), np.zeros(3, np.float32), 1, 1.0) == 18


def test_moe_combine_order_on_tiny_f32_free_case():
    # moe.rs:331-336: out = 0; += c_e * expert_e (ascending ID); += 1.0 * shared.
    # Checked against an independent numpy restatement on IQ2_S/IQ3_S experts.
    rng = np.random.default_rng(11)
    hidden, ffn = 256, 256

    def iq2(rows, cols):
        w = rng.integers(0, 256, size=rows * cols // 256 * 82, dtype=np.uint8)
        for b in range(rows * cols // 256):
            w[b * 82 : b * 82 + 2] = np.frombuffer(np.float16(rng.uniform(0.001, 0.01)).tobytes(), np.uint8)
        return w

    def iq3(rows, cols):
        w = rng.integers(0, 256, size=rows * cols // 256 * 110, dtype=np.uint8)
        for b in range(rows * cols // 256):
            w[b * 110 : b * 110 + 2] = np.frombuffer(np.float16(rng.uniform(0.001, 0.01)).tobytes(), np.uint8)
        return w

    experts = [
        (orc.TYPE_IQ2_S, iq2(ffn, hidden), orc.TYPE_IQ2_S, iq2(ffn, hidden), orc.TYPE_IQ3_S, iq3(hidden, ffn), hidden, ffn)
        for _ in range(4)
    ]
    shared = (orc.TYPE_IQ2_S, iq2(ffn, hidden), orc.TYPE_IQ2_S, iq2(ffn, hidden), orc.TYPE_IQ3_S, iq3(hidden, ffn), hidden, ffn)
    table = orc.ExpertTable(experts, shared)
    x = rng.standard_normal(hidden).astype(np.float32)
    ids = np.array([1, 3], np.uint32)
    coefs = np.array([0.25, 0.75], np.float32)
    out = orc.moe_routed(table, ids, coefs, x, preflight=True)
    out1 = orc.moe_routed(table, ids, coefs, x, preflight=False)
    np.testing.assert_array_equal(out.view(np.uint32), out1.view(np.uint32))

    def expert_out(e):
        gty, gb, uty, ub, dty, db, _, _ = e
        g, _ = orc.gemv(gty, hidden, ffn, gb, x)
        u, _ = orc.gemv(uty, hidden, ffn, ub, x)
        h = orc.swiglu(g, u)
        d, _ = orc.gemv(dty, ffn, hidden, db, h)
        return d

    want = np.zeros(hidden, np.float32)
    for i, c in zip(ids, coefs):
        want = (want + np.float32(c) * expert_out(experts[i])).astype(np.float32)
    want = (want + np.float32(1.0) * expert_out(shared)).astype(np.float32)
    np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))
