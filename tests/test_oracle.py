"""The oracle (oracle/attn_oracle.c) pinned against the reference's own attention.

Pins, all bit-exact (the restatement does the same double-precision operations in the same order):
  * golden vectors in tests/golden/ made by the reference's compiled cpu/forward_cpu.c attention();
  * the reference's attention() itself (oracle/_ref/libref_cpu.so), when it has been built;
  * decode attention (cuda/kvcache.cu:88-129 restated) of query i over keys 0..i == prefill row i.
"""
import hashlib
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _ref_cpu():
    try:
        return O.RefCPU()
    except FileNotFoundError:
        pytest.skip("reference CPU attention not built (make -C oracle ref needs the reference tree)")


def test_golden_T40_bit_exact(oracle):
    g = np.load(os.path.join(GOLD, "prefill_T40.npz"))
    qkv = g["qkv_f16"].view(np.float16).astype(np.float32)
    assert np.array_equal(oracle.prefill(qkv), g["att"])


def test_golden_config1_T128_bit_exact(oracle):
    g = np.load(os.path.join(GOLD, "prefill_T128_cfg1.npz"))
    qkv = O.seeded_qkv(int(g["seed"]), int(g["T"]))
    sha = hashlib.sha256(qkv.astype(np.float16).tobytes()).hexdigest()
    assert sha == g["qkv_f16_sha256"].item().decode(), "seeded input generator drifted"
    assert np.array_equal(oracle.prefill(qkv), g["att"])


def test_golden_fixtures_reproduced_by_the_reference():
    """The committed fixtures are what the reference's own compiled attention() returns today."""
    ref = _ref_cpu()
    g = np.load(os.path.join(GOLD, "prefill_T40.npz"))
    assert np.array_equal(ref.prefill(g["qkv_f16"].view(np.float16).astype(np.float32)), g["att"])
    g = np.load(os.path.join(GOLD, "prefill_T128_cfg1.npz"))
    assert np.array_equal(ref.prefill(O.seeded_qkv(int(g["seed"]), int(g["T"]))), g["att"])


@pytest.mark.parametrize("T", [1, 2, 31, 32, 33, 127, 128, 129, 161, 300])
def test_oracle_equals_reference_cpu(oracle, T):
    ref = _ref_cpu()
    qkv = O.seeded_qkv(1000 + T, T)
    assert np.array_equal(oracle.prefill(qkv), ref.prefill(qkv))


def test_oracle_equals_reference_cpu_max_ctx(oracle):
    ref = _ref_cpu()
    qkv = O.seeded_qkv(77, O.N_CTX)
    assert np.array_equal(oracle.prefill(qkv), ref.prefill(qkv))


def _cache_from_qkv(oracle, qkv_f32, max_t):
    """One layer's [H, maxT, D] K/V slabs filled by the restated scatter (cuda/kvcache.cu:67-76)."""
    u16 = qkv_f32.astype(np.float16).view(np.uint16)
    k = np.zeros((O.H, max_t, O.D), np.uint16)
    v = np.zeros((O.H, max_t, O.D), np.uint16)
    oracle.kv_scatter(k, v, np.ascontiguousarray(u16))
    return k.view(np.float16).astype(np.float32), v.view(np.float16).astype(np.float32)


def test_decode_equals_prefill_rows_golden(oracle):
    g = np.load(os.path.join(GOLD, "prefill_T40.npz"))
    qkv = g["qkv_f16"].view(np.float16).astype(np.float32)
    k, v = _cache_from_qkv(oracle, qkv, max_t=48)
    for i in range(qkv.shape[0]):
        got = oracle.decode(qkv[i, :O.E], k, v, i + 1)
        assert np.array_equal(got, g["att"][i]), f"row {i}"


def test_decode_equals_prefill_rows_long(oracle):
    T = 700
    qkv = O.seeded_qkv(5, T)
    att = oracle.prefill(qkv)
    k, v = _cache_from_qkv(oracle, qkv, max_t=1024)
    for i in (0, 1, 63, 64, 65, 255, 511, 699):
        assert np.array_equal(oracle.decode(qkv[i, :O.E], k, v, i + 1), att[i]), f"row {i}"


def test_scatter_layout_matches_reference_formula(oracle):
    """K[h][pos][d] = qkv[pos][E + h*D + d], V likewise at 2E (cuda/kvcache.cu:67-76)."""
    T, max_t = 5, 9
    u16 = np.arange(T * O.QKV, dtype=np.uint32).astype(np.uint16).reshape(T, O.QKV)
    k = np.zeros((O.H, max_t, O.D), np.uint16)
    v = np.zeros((O.H, max_t, O.D), np.uint16)
    oracle.kv_scatter(k, v, u16, pos0=3)
    for t in range(T):
        for h in (0, 7, 11):
            assert np.array_equal(k[h, 3 + t], u16[t, O.E + h * O.D:O.E + (h + 1) * O.D])
            assert np.array_equal(v[h, 3 + t], u16[t, 2 * O.E + h * O.D:2 * O.E + (h + 1) * O.D])
    assert not k[:, :3].any() and not k[:, 8:].any()


def test_oracle_rejects_bad_arguments(oracle):
    with pytest.raises(ValueError):
        oracle.decode(np.zeros(768, np.float32), np.zeros((12, 4, 64), np.float32),
                      np.zeros((12, 4, 64), np.float32), 5)
    with pytest.raises(ValueError):
        oracle.decode(np.zeros(768, np.float32), np.zeros((12, 4, 64), np.float32),
                      np.zeros((12, 4, 64), np.float32), 0)
