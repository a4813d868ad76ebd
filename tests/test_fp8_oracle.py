"""The oracle's FP8 E4M3 weight format (CPU): the encoder against torch's
float8_e4m3fn conversion (an independent implementation of the OCP E4M3
format, round to nearest even) over every finite BF16 value in range, the
saturation rule, the decoder over all 256 codes, the power-of-two row scales,
and that every dequantized weight is exactly a BF16 value.
"""
import numpy as np
import pytest

from gpu_util import bf


def _all_bf16():
    b = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    v = bf(b)
    return b[np.isfinite(v)], v[np.isfinite(v)]


def test_e4m3_encoder_matches_torch_in_range(oracle):
    import torch

    _, v = _all_bf16()
    v = v[np.abs(v) <= 448.0]
    mine = np.array([oracle.e4m3(float(x)) for x in v], np.uint8)
    ref = torch.from_numpy(v.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    bad = mine != ref
    assert not bad.any(), (v[bad][:8], mine[bad][:8], ref[bad][:8])


def test_e4m3_saturates_and_keeps_sign(oracle):
    for x in (448.0, 449.0, 464.0, 480.0, 1e6, 3.0e38):
        assert oracle.e4m3(x) == 0x7E
        assert oracle.e4m3(-x) == 0xFE
    assert oracle.e4m3(0.0) == 0x00 and oracle.e4m3(-0.0) == 0x80
    assert oracle.e4m3(float("nan")) & 0x7F == 0x7F
    # ties to even at the subnormal and normal steps
    assert oracle.e4m3(2.0 ** -10) == 0x00 and oracle.e4m3(3 * 2.0 ** -10) == 0x02
    assert oracle.e4m3(1.0625) == 0x38 and oracle.e4m3(1.1875) == 0x3A


def test_e4m3_decoder_all_codes(oracle):
    import torch

    codes = np.arange(256, dtype=np.uint8)
    mine = np.array([oracle.e4m3_value(int(c)) for c in codes], np.float32)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(ref)
    assert (np.isnan(mine) == nan).all()
    np.testing.assert_array_equal(mine[~nan], ref[~nan])
    # encode(decode(c)) == c for every finite code
    for c in codes[~nan]:
        assert oracle.e4m3(float(mine[c])) == c


@pytest.mark.parametrize("cols", [16, 1024, 4096 + 32])
def test_quantize_rows_scale_rule_and_exact_bf16(oracle, cols):
    rng = np.random.default_rng(cols)
    rows = 64
    w = (rng.standard_normal((rows, cols)) * np.exp2(rng.integers(-20, 12, (rows, 1)))).astype(np.float32)
    w[3] = 0.0                         # all-zero row: scale 1, codes 0
    w[5] = rng.uniform(-20.0, 20.0, cols)
    w[5, 7] = 448.0 * 2.0 ** -4        # a row whose maximum lands exactly on 448 * 2^e
    wb = (w.view(np.uint32) >> 16).astype(np.uint16)  # truncate to BF16 bits
    q, sc = oracle.quantize_e4m3(wb)
    e = np.log2(sc)
    assert np.all(e == np.round(e)), "scales are powers of two"
    mx = np.abs(bf(wb)).max(axis=1)
    nz = mx > 0
    # smallest e with max <= 448 * 2^e
    assert np.all(mx[nz] <= 448.0 * sc[nz]) and np.all(mx[nz] > 224.0 * sc[nz])
    assert sc[3] == 1.0 and not q[3].any()
    assert sc[5] == 2.0 ** -4 and q[5, 7] == 0x7E
    # dequantized values: exactly representable in BF16 (<= 4 significant bits)
    deq = np.array([oracle.e4m3_value(int(c)) for c in range(256)], np.float32)[q] * sc[:, None]
    back = bf((deq.view(np.uint32) >> 16).astype(np.uint16))
    np.testing.assert_array_equal(back, deq)
    # and within half an E4M3 step of the weights (relative to the row scale)
    err = np.abs(deq - bf(wb)) / sc[:, None]
    assert np.all(err <= np.maximum(2.0 ** -10, np.abs(bf(wb)) / sc[:, None] * 2.0 ** -4) * 1.0001)


def test_oracle_fp8_model_is_close_to_bf16(oracle):
    """An FP8-weight model (every GEMV matrix replaced by its E4M3 round trip)
    stays close to the BF16 model: same greedy tokens on most steps, logits
    highly correlated."""
    from oracle import ModelConfig

    cfg = ModelConfig.make(256, 512, 2, 4, 2, 128, 4096, 64, tied=True)
    a = oracle.model(cfg, seed=3)
    b = oracle.model(cfg, seed=3).quantize_fp8()
    toks = oracle.prompt_ids(24, seed=5, vocab=4096)
    agree = 0
    for t in toks:
        na, nb = a.forward(int(t)), b.forward(int(t))
        la, lb = bf(a.logits()).astype(np.float64), bf(b.logits()).astype(np.float64)
        assert la @ lb / (np.linalg.norm(la) * np.linalg.norm(lb)) > 0.98
        assert not np.array_equal(la, lb)
        agree += int(na == nb)
    assert agree >= len(toks) // 2
    a.close()
    b.close()



@pytest.mark.parametrize("n,k,sms", [(300, 320, 148), (37, 64, 4), (4096, 192, 148), (66, 512, 7)])
def test_packed_fp8_layout_is_a_tiled_bijection(n, k, sms):
    """q3_e4m3_packed_offset (the FP8 GEMV's weight layout, the same function
    the device packer, quantizer and BF16 expansion use): every weight has its
    own byte inside q3_e4m3_packed_bytes, each 16-column group is 16 contiguous
    bytes, and each 16-row x
    256-column tile of a CTA's row band is one contiguous run of rows x 256
    bytes (one bulk copy)."""
    from inference_b200 import lib

    L = lib()
    size = L.q3_e4m3_packed_bytes(n, k)
    off = np.array([[L.q3_e4m3_packed_offset(n, k, sms, r, c) for c in range(k)] for r in range(n)], np.int64)
    assert off.max() < size and off.min() >= 0
    assert len(np.unique(off)) == n * k
    assert (off[:, 1::2] == off[:, ::2] + 1).all()
    # each 16-column group is 16 contiguous bytes (the packer and the BF16 expansion
    # of the FP8 prefill move whole groups)
    for j in range(1, 16):
        assert (off[:, j::16] == off[:, 0::16][:, :off[:, j::16].shape[1]] + j).all()
    # tiles: the 16-byte groups of one row segment of 256 columns sit in one
    # 256-byte row of the tile, each tile's rows back to back
    base = off[:, ::16] & ~255
    for c0 in range(0, k, 256):
        blk = base[:, c0 // 16:(c0 + 256) // 16]
        assert (blk == blk[:, :1]).all()
    assert L.q3_e4m3_packed_offset(n, k, sms, n, 0) == 2**64 - 1  # out of range
