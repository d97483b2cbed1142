"""Standalone codec seams on the GPU, bit-exact against the CPU checker.

The reference swaps these functions as units (``_decode`` / ``_encode`` at
costate.py:393-395, ``decompress_v`` at oneq.py:51-67), so each C-ABI seam
must equal the checker bit for bit on its own, not only inside the fused
step:

* ``ta_v_decode``       -- decompress_v / dequantize_logscale_nbits
                           (quantize.py:183-214); also within 1 ulp of the
                           reference's own output (torch's exp);
* ``ta_costate_decode`` -- decode_blocks (costate.py:261-323);
* ``ta_costate_encode`` -- encode_blocks + _pack_signs (costate.py:157-258).
"""
import numpy as np
import pytest
import torch

import golden_util as GU

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def to_np(t):
    return t.detach().cpu().numpy()


def bits16(t):
    return to_np(t.contiguous().view(torch.int16)).view(np.uint16)


def _ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


def _decode(idx, hdr_bits, n, nbits):
    from turboadam_b200.oneq import decompress_v

    cv = {"indices": cuda(idx), "scales": cuda(hdr_bits.view(np.float16)).reshape(-1, 2),
          "n_bits": nbits, "original_shape": torch.Size([n]), "original_length": n,
          "block_size": 128}
    return to_np(decompress_v(cv))


def test_v_decode_reference_golden(oracle):
    """Every v_bits, n in {1, 129, 16421}: equal to the checker, within 1 ulp
    of the reference's decompress_v."""
    d = GU.load("v_decode.npz")
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        nbits, n = (int(x) for x in d[k + "_meta"])
        idx, hdr = d[f"{k}_idx"], d[f"{k}_hdr"].reshape(-1)
        v = _decode(idx, hdr, n, nbits)
        ov = oracle.v_decode(idx, hdr, n, nbits)
        np.testing.assert_array_equal(v.view(np.uint32), ov.view(np.uint32), err_msg=k)
        assert _ulps(v, d[f"{k}_v"]).max() <= 1, k


@pytest.mark.parametrize("nbits", [2, 3, 4, 6, 8])
@pytest.mark.parametrize("n", [77, 128 * 4096 + 37])
def test_v_decode_evolved_states(oracle, nbits, n):
    """States produced by 1Q updates (wide spans, constant blocks, zero
    gradients), including headers at the fp16 extremes."""
    rng = np.random.default_rng(nbits * 7 + n)
    idx, hdr = oracle.v_init(n)
    B = (n + 127) // 128
    for s in range(2):
        g = (rng.standard_normal(n) * 10.0 ** rng.uniform(-7, 0, n)).astype(np.float32)
        g[rng.random(n) < 0.05] = 0.0
        idx, hdr, _ = oracle.v_update(idx, hdr, g, nbits, 0.999, rng.random(B * 128, np.float32))
    hdr = hdr.copy()
    hdr[:4] = np.array([0xFBFF, 0xFBFF, 0x7BFF, 0x7BFF], np.uint16)[: min(4, hdr.size)]
    v = _decode(idx, hdr, n, nbits)
    ov = oracle.v_decode(idx, hdr, n, nbits)
    np.testing.assert_array_equal(v.view(np.uint32), ov.view(np.uint32))


def _encoding(rng, n):
    B = (n + 127) // 128
    labels = rng.integers(0, 3, B).astype(np.uint8)
    signs = rng.integers(0, 256, (n + 7) // 8).astype(np.uint8)
    norms = (rng.random(B) * 10.0 ** rng.uniform(-8, 2, B)).astype(np.float32)
    norms[rng.random(B) < 0.05] = 0.0
    amp = (norms / np.float32(np.sqrt(128.0))).astype(np.float16).view(np.uint16)
    return labels, signs, norms, amp


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [300, 4096, 65536 + 37])
def test_costate_decode_bitexact(oracle, n, dtype):
    from turboadam_b200.costate import decode_blocks

    rng = np.random.default_rng(n)
    labels, signs, norms, amp = _encoding(rng, n)
    g = torch.from_numpy((rng.standard_normal(n) * 1e-3).astype(np.float32)).to(dtype)
    alpha = np.float32(rng.standard_normal() * 0.1)
    enc = {"labels": cuda(labels), "sign_packed": cuda(signs), "block_norms": cuda(norms),
           "scales": cuda(amp.view(np.float16))}
    m = decode_blocks(enc, float(alpha), g.cuda(), 128, n)
    om = oracle.costate_decode(labels, signs, norms, amp, alpha, to_np(g.float()))
    np.testing.assert_array_equal(to_np(m).view(np.uint32), om.view(np.uint32))


@pytest.mark.parametrize("n", [1, 300, 4096, 65536 + 37])
def test_costate_encode_bitexact(oracle, n):
    from turboadam_b200.costate import encode_blocks

    rng = np.random.default_rng(n + 1)
    delta = (rng.standard_normal(n) * 10.0 ** rng.uniform(-9, 1, n)).astype(np.float32)
    delta[rng.random(n) < 0.05] = 0.0
    delta[rng.random(n) < 0.02] = -0.0  # -0 is not < 0: its sign bit stays clear
    B = (n + 127) // 128
    enc = encode_blocks(cuda(delta), torch.zeros(B, dtype=torch.uint8, device="cuda"))
    osg, onrm, oamp = oracle.costate_encode(delta)
    np.testing.assert_array_equal(to_np(enc["sign_packed"]), osg)
    np.testing.assert_array_equal(to_np(enc["block_norms"]).view(np.uint32), onrm.view(np.uint32))
    np.testing.assert_array_equal(bits16(enc["scales"]), oamp)


def test_costate_codec_round_trip_reference_golden(oracle):
    """The reference's own encodings (costate.npz): decoding them on the GPU
    with the reference's alpha equals the checker's decode bit for bit."""
    from turboadam_b200.costate import decode_blocks

    d = GU.load("costate.npz")
    for c in range(int(d["n_cases"][0])):
        k = f"c{c:03d}"
        n, ns = (int(x) for x in d[k + "_meta"])
        for s in range(ns - 1):  # the encoding of step s decodes with step s + 1's gradient
            lab, sg = d[f"{k}_s{s}_labels"], d[f"{k}_s{s}_signs"]
            nr, am = d[f"{k}_s{s}_norms"], d[f"{k}_s{s}_amp"]
            alpha = d[f"{k}_s{s}_alpha"][0]
            g = d[f"{k}_s{s + 1}_g"]
            enc = {"labels": cuda(lab), "sign_packed": cuda(sg), "block_norms": cuda(nr),
                   "scales": cuda(am.view(np.float16))}
            m = decode_blocks(enc, float(alpha), cuda(g), 128, n)
            om = oracle.costate_decode(lab, sg, nr, am, alpha, g)
            np.testing.assert_array_equal(to_np(m).view(np.uint32), om.view(np.uint32),
                                          err_msg=f"{k} s{s}")
