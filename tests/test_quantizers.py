"""The device quantizers and 1-bit packers (retrieve_b200/quantize.py over
rb_quantize_int8_global, rb_pack_signs and rb_quantize_int8) against the oracle
and the fixture the reference's own quantizers produced
(tests/golden/golden_quant.npz)."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import bits, knn
from retrieve_b200 import _lib

QUANT = np.load(Path(__file__).resolve().parent / "golden" / "golden_quant.npz")


def _q():
    from retrieve_b200 import quantize

    return quantize


def test_capi_argument_checks_need_no_device():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.rb_quantize_int8_global_workspace_size(ctypes.byref(n)) == 0 and n.value >= 4
    assert lib.rb_quantize_int8_global(None, 10, 0, None, 0, None, None, None, 0, None) == _lib.RB_ERR_INVALID_ARG
    assert lib.rb_quantize_int8_global(None, 10, 8, None, 0, None, None, None, 0, None) == _lib.RB_ERR_WORKSPACE
    assert lib.rb_pack_signs(None, 4, 100, None, None) == _lib.RB_ERR_INVALID_ARG  # D not a multiple of 64
    assert lib.rb_pack_signs(None, 4, 128, None, None) == _lib.RB_ERR_INVALID_ARG  # null pointers
    assert lib.rb_pack_signs(None, 0, 128, None, None) == _lib.RB_OK  # nothing to pack


def test_cpu_tensors_raise():
    q = _q()
    with pytest.raises(ValueError):
        q.pack_signs(torch.zeros(2, 64))
    with pytest.raises(ValueError):
        q.quantize_int8_global(torch.zeros(2, 64))


@pytest.mark.gpu
def test_quantize_int8_global_matches_reference_and_oracle():
    q = _q()
    x = torch.from_numpy(QUANT["global_x"]).cuda()
    codes, scale = q.quantize_int8_global(x)
    assert np.array_equal(codes.cpu().numpy(), QUANT["global_codes"])
    _, want = knn.quantize_int8_global(QUANT["global_x"])
    assert np.float32(scale) == np.float32(want)
    # the device form is torch's own: abs_max (a 0-dim CUDA tensor) / 127.0
    am = torch.maximum(x.amax(), -x.amin()).clamp(min=1e-8)
    assert np.float32(scale) == np.float32((am / 127.0).item())
    perm = torch.from_numpy(QUANT["global_perm"]).cuda()
    codes_p, scale_p = q.quantize_int8_global(x, rows=perm)
    assert np.array_equal(codes_p.cpu().numpy(), QUANT["global_codes_perm"]) and scale_p == scale
    codes_n, scale_n = q.quantize_int8_global(torch.from_numpy(QUANT["global_nan_x"]).cuda())
    assert np.isnan(scale_n) and np.array_equal(codes_n.cpu().numpy(), QUANT["global_nan_codes"])
    with pytest.raises(IndexError):
        q.quantize_int8_global(x, rows=torch.tensor([0, 1000], device="cuda"))


@pytest.mark.gpu
def test_quantize_int8_global_large_table():
    """A table spread over many CTAs (the abs-max fold) with the maximum in the last row."""
    q = _q()
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(300_000, 128, generator=g, device="cuda")
    x[-1, -1] = -50.0
    codes, scale = q.quantize_int8_global(x)
    am = torch.maximum(x.amax(), -x.amin())
    assert float(am) == 50.0 and np.float32(scale) == np.float32((am / 127.0).item())
    want = (x / am * 127.0).round().clamp(-128, 127).to(torch.int8)  # the reference's expression on CUDA
    assert torch.equal(codes, want)


@pytest.mark.gpu
def test_quantize_int8_nan_and_inf_rows():
    q = _q()
    x = QUANT["q8_special_x"]
    codes, scales = q.quantize_int8(torch.from_numpy(x).cuda())
    assert np.array_equal(codes.cpu().numpy(), QUANT["q8_special_codes"])
    want_c, want_s = knn.quantize_int8(x)
    assert np.array_equal(codes.cpu().numpy(), want_c)
    assert np.array_equal(scales.cpu().numpy(), want_s, equal_nan=True)


@pytest.mark.gpu
def test_pack_signs_matches_reference():
    q = _q()
    v = torch.from_numpy(QUANT["pack_values"]).cuda()
    assert np.array_equal(q.pack_signs(v).cpu().numpy(), QUANT["pack_words"])
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randn(3, 777, 512, generator=g, device="cuda")
    w[0, 0, :128] = 0.0
    got = q.pack_signs(w)
    assert got.shape == (3, 777, 8)
    assert np.array_equal(got.cpu().numpy(), bits.pack_signs(w.cpu().numpy()))


@pytest.mark.gpu
def test_simhash_and_oporp_builds():
    """The 1-bit builds on the device: the projections are the reference's torch calls on
    the same device, the packing is the kernel; the words equal the oracle's packing of
    the same projected values, and agree with the reference's CPU build except where a
    projected value sits within the GEMMs' rounding of zero."""
    q = _q()
    embs = torch.from_numpy(QUANT["sim_embs"]).cuda()
    query = torch.from_numpy(QUANT["sim_query"]).cuda()
    codes, r = q.quantize_simhash_1bit(embs, 512, seed=3)
    assert np.array_equal(codes.cpu().numpy(), bits.pack_signs((embs @ r.t()).cpu().numpy()))
    qb = q.project_simhash_1bit_query(query, r)
    assert np.array_equal(qb.cpu().numpy(), bits.pack_signs((query @ r.t()).cpu().numpy()))
    r_ref = torch.from_numpy(QUANT["sim_r"]).cuda()
    ours = q.project_simhash_1bit_query(embs, r_ref).cpu().numpy()
    diff = np.bitwise_count((ours ^ QUANT["sim_bits"]).view(np.uint64)).sum()
    assert diff <= 0.001 * ours.size * 64
    obits, signs, perm = q.quantize_oporp_1bit(embs, seed=5)
    proj = (embs * signs.to(embs.dtype)).index_select(1, perm)
    assert np.array_equal(obits.cpu().numpy(), bits.pack_signs(proj.cpu().numpy()))
    signs_ref = torch.from_numpy(QUANT["oporp_signs"]).cuda()
    perm_ref = torch.from_numpy(QUANT["oporp_perm"]).cuda()
    oq = q.project_oporp_1bit_query(query, signs_ref, perm_ref)
    assert np.array_equal(oq.cpu().numpy(), QUANT["oporp_qbits"])  # k_bits = D: no sums, exact
