"""The oracle's NVFP4 weight format (oracle/q3_oracle.c): E2M1 values, E4M3
scales per 16-column block, power-of-two row scales.  Known answers for the
encoders, the exactness of the dequantized weights as BF16 values, and the
error bound of a block."""
import numpy as np
import pytest

from inputs import uniform_bf16


@pytest.mark.parametrize("x,code", [(0.0, 0), (0.25, 0), (0.26, 1), (0.5, 1), (0.75, 2), (1.25, 2), (1.3, 3),
                                    (1.75, 4), (2.5, 4), (2.6, 5), (3.5, 6), (5.0, 6), (5.1, 7), (6.0, 7), (1e9, 7),
                                    (-1.0, 0xA), (-0.1, 0x8), (-7.0, 0xF)])
def test_e2m1_encoder(oracle, x, code):
    """Nearest, ties to the even code, saturating at 6."""
    assert oracle.e2m1(x) == code


def test_e2m1_values(oracle):
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for c in range(16):
        v = oracle.e2m1_value(c)
        assert abs(v) == mags[c & 7] and (v < 0) == (c >= 8 and c != 8)


def test_nvfp4_known_row(oracle):
    """A row of sixteen 1.0: row scale 2^-11, block scale E4M3(1/6 * 2^11 = 341.3) = 352
    (code 0x7B), values E2M1(2048 / 352 = 5.82) = 6 -> each weight dequantizes to
    6 * 352 * 2^-11 = 1.03125."""
    w = np.full((1, 16), 0x3F80, np.uint16)  # BF16 1.0
    q, bs, rs = oracle.quantize_nvfp4(w)
    assert rs[0] == 2.0 ** -11
    assert bs[0, 0] == 0x7B and oracle.e4m3_value(0x7B) == 352.0
    assert (q == 7).all()


def _bf(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_nvfp4_dequantized_weights_are_bf16_and_close(oracle):
    w = uniform_bf16(1234, (37, 256))
    q, bs, rs = oracle.quantize_nvfp4(w)
    e2 = np.vectorize(oracle.e2m1_value)(q).astype(np.float64)
    s = np.vectorize(oracle.e4m3_value)(bs).astype(np.float64)
    deq = e2 * np.repeat(s, 16, axis=1) * rs[:, None].astype(np.float64)
    # exact BF16 values: the round trip through BF16 bits changes nothing
    as_bf = _bf((deq.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)).astype(np.float64)
    np.testing.assert_array_equal(as_bf, deq)
    x = _bf(w).astype(np.float64)
    amax = np.repeat(np.abs(x).reshape(37, 16, 16).max(axis=2), 16, axis=1)
    assert (np.abs(deq - x) <= 0.25 * amax + 1e-30).all()
    # every block scale fits E4M3 (no saturation at 448)
    assert (s <= 448.0).all()


@pytest.mark.parametrize("n,k,sms", [(300, 512, 148), (37, 64, 4), (4096, 192, 148), (66, 1024, 7), (19, 2560, 3)])
def test_packed_nvfp4_layout_is_a_tiled_bijection(n, k, sms):
    """q3_nvfp4_packed_offset (the NVFP4 GEMV's weight layout, the same
    functions the device quantizer and expansion use): every pair of columns
    has its own byte and every 16-column block its own scale byte, all inside
    q3_nvfp4_packed_bytes; a block's nibbles are 8 contiguous bytes; and each
    16-row x 512-column item of a CTA's row band is one contiguous run of
    rows x 288 bytes (one bulk copy), nibbles first, scales after."""
    from inference_b200 import lib

    L = lib()
    size = L.q3_nvfp4_packed_bytes(n, k)
    assert size == n * ((k + 511) // 512) * 288
    nib = np.array([[L.q3_nvfp4_packed_offset(n, k, sms, r, c, 0) for c in range(0, k, 2)] for r in range(n)],
                   np.int64)
    sc = np.array([[L.q3_nvfp4_packed_offset(n, k, sms, r, c, 1) for c in range(0, k, 16)] for r in range(n)],
                  np.int64)
    every = np.concatenate([nib.ravel(), sc.ravel()])
    assert every.min() >= 0 and every.max() < size
    assert len(np.unique(every)) == every.size  # nibble and scale bytes all distinct
    # a column and its odd neighbour share a byte
    assert L.q3_nvfp4_packed_offset(n, k, sms, 0, 1, 0) == L.q3_nvfp4_packed_offset(n, k, sms, 0, 0, 0)
    # a 16-column block: 8 contiguous bytes
    for j in range(1, 8):
        assert (nib[:, j::8] == nib[:, 0::8][:, :nib[:, j::8].shape[1]] + j).all()
    # items: the bytes of rows sharing a tile and a 512-column chunk form one contiguous run
    used = np.zeros(size, bool)
    used[every] = True
    assert used[: n * (k // 512) * 288].all() if k % 512 == 0 else True
    assert L.q3_nvfp4_packed_offset(n, k, sms, n, 0, 0) == 2**64 - 1  # out of range
