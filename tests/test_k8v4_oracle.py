"""The K8/V4 restatement (oracle/k8v4.py) and the host side of its path, on
the CPU.

The reader is pinned to the reference's own gate expression for it
(docs/superpowers/plans/2026-09-08-direct-k8v4-attention.md:62-72): every
K8 code 0..255 and V4 code 0..15, with scales 0 / small / 1 / large finite,
must dequantise exactly to ((codes.float() - midpoint) * (scales.float() /
2 ** (bits - 1))).half().  The bit-plane packing and the writer are
third-party (ExLlamaV3, absent): they are checked for self-consistency and
for the quantiser's error bound, not against reference output.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import k8v4, rng
from oracle.attention import attention_fp32
from tests.golden import cases

SCALES = np.array([0.0, 2.0 ** -24, 6.1e-5, 0.0078125, 0.37, 1.0, 3.5, 1000.0, 65504.0], dtype=np.float16)


def _plan_gate(codes: torch.Tensor, scales: torch.Tensor, bits: int) -> torch.Tensor:
    midpoint = 2 ** (bits - 1) - 0.5
    return ((codes.float() - midpoint) * (scales.float() / 2 ** (bits - 1))).half()


@pytest.mark.parametrize("bits", [8, 4])
def test_reader_matches_the_reference_gate_on_every_code_and_scale(bits):
    codes = np.arange(1 << bits, dtype=np.uint8)
    # the oracle takes [..., 32] blocks; lay the codes out in blocks of 32
    blocks = np.resize(codes, (SCALES.size, 256))
    got = k8v4.dequant(blocks.reshape(SCALES.size, 8, 32), np.repeat(SCALES[:, None], 8, 1), bits)
    ref = _plan_gate(torch.from_numpy(blocks.reshape(SCALES.size, 8, 32).astype(np.int64)),
                     torch.from_numpy(np.repeat(SCALES[:, None, None], 8, 1)), bits)
    assert np.array_equal(got.view(np.uint16), ref.numpy().view(np.uint16))


@pytest.mark.parametrize("bits", [8, 4])
def test_bit_planes_round_trip(bits):
    codes = (rng.bytes_(11, 64 * 32).astype(np.int32) % (1 << bits)).astype(np.uint8).reshape(64, 32)
    words = k8v4.pack_planes(codes, bits)
    assert words.shape == (64, bits) and words.dtype == np.uint32
    assert np.array_equal(k8v4.unpack_planes(words, bits), codes)
    # word i holds bit i of code t at bit t
    t, i = 5, bits - 1
    assert ((int(words[0, i]) >> t) & 1) == ((int(codes[0, t]) >> i) & 1)


def test_butterfly_is_the_hadamard_rotation():
    R = k8v4.hadamard32().astype(np.float64)
    assert np.abs(R @ R.T - np.eye(32)).max() < 1e-6
    assert np.array_equal(R, R.T)
    x = rng.normal(3, 40 * 32).reshape(40, 32).astype(np.float32)
    assert np.abs(k8v4.rotate_butterfly(x) - x.astype(np.float64) @ R.T).max() < 1e-5


@pytest.mark.parametrize("bits", [8, 4])
def test_writer_error_bound_and_scale(bits):
    x = cases.kv_rows(21, 64, 4).astype(np.float16).astype(np.float32).reshape(-1, 32)
    xr = k8v4.rotate_butterfly(x)
    codes, scales = k8v4.quantize_blocks(xr, bits)
    assert np.array_equal(scales, np.minimum(np.abs(xr).max(-1), 65504).astype(np.float16))
    y = k8v4.dequant(codes, scales, bits).astype(np.float64)
    s = scales.astype(np.float64)[:, None]
    m = 2 ** (bits - 1)
    # half a bin, plus the scale's own FP16 rounding and the FP16 reconstruction
    bound = s / m * 0.5 + s * 2.0 ** -10 + np.abs(y) * 2.0 ** -11 + 1e-12
    assert (np.abs(y - xr) <= bound).all()
    zero, zs = k8v4.quantize_blocks(np.zeros((2, 32), np.float32), bits)
    assert (zero == m).all() and (zs == 0).all()
    assert (k8v4.dequant(zero, zs, bits) == 0).all()


def test_writing_no_rows_is_a_no_op():
    cache = k8v4.empty_cache(1)
    k8v4.write_rows(cache, np.zeros((0, 4, 256), np.float32), np.zeros((0, 4, 256), np.float32), np.array([0]), 5)
    assert not cache["k_cache"].any() and not cache["v_scales"].any()


def test_rotated_attention_equals_attention_over_restored_rows():
    P, L, S = 3, 600, 7
    table = rng.permutation(5, P)
    cache = k8v4.empty_cache(P)
    k = cases.kv_rows(2, L, 4).astype(np.float32)
    v = cases.kv_rows(3, L, 4).astype(np.float32)
    k8v4.write_rows(cache, k, v, table, 0)
    q = torch.from_numpy(rng.normal(4, S * 24 * 256).reshape(S, 24, 256).astype(np.float32)).half()
    a = k8v4.attention(q, cache, table, L - S)
    b = k8v4.attention_rotated(q, cache, table, L - S)
    assert (a - b).abs().max().item() < 1e-5 * max(1.0, a.abs().max().item())
    # the 8-bit keys and 4-bit values keep the output near the unquantised one
    exact = attention_fp32(q.float(), torch.from_numpy(k), torch.from_numpy(v), 1 / 16, L - S)
    assert ((a - exact).norm() / exact.norm()).item() < 0.15


def test_host_module_matches_the_oracle_geometry():
    from qwarz_b200 import k8v4 as host

    assert np.array_equal(host.hadamard32().numpy(), k8v4.hadamard32())
    kc, vc, ks, vs = host.empty_cache(2, "cpu")
    ref = k8v4.empty_cache(2)
    assert kc.shape == ref["k_cache"].shape and vc.shape == ref["v_cache"].shape
    assert ks.shape == ref["k_scales"].shape and ks.dtype == torch.float16
    assert host.check_cache(kc, vc, ks, vs) == 2
    with pytest.raises(ValueError, match="Packed cache geometry"):
        host.check_cache(kc, kc, ks, vs)
    with pytest.raises(ValueError, match="scales"):
        host.check_cache(kc, vc, ks.float(), vs)
    with pytest.raises(ValueError, match="CUDA"):
        host.append(torch.zeros(1, 4, 256, dtype=torch.half), torch.zeros(1, 4, 256, dtype=torch.half),
                    (kc, vc, ks, vs), torch.zeros(1, 2, dtype=torch.int32), torch.zeros(1, dtype=torch.int32))
