"""The FP8 activation quantiser's CPU restatement (oracle/moe_oracle.py: quantize_hidden,
encode_e4m3) against torch's float8_e4m3fn cast, and its edge cases. The device quantiser is
compared with it bit for bit in tests/test_gpu_quant.py."""
import numpy as np
import torch


def test_encoder_roundtrips_every_finite_code(oracle):
    vals = oracle._e4m3_table()
    codes = np.where(np.isfinite(vals))[0].astype(np.uint8)
    np.testing.assert_array_equal(oracle.encode_e4m3(vals[codes]), codes)


def test_encoder_ties_to_even_and_saturates(oracle):
    vals = oracle._e4m3_table()[:127].astype(np.float64)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)      # exact midpoints (fp32-representable)
    got = oracle.encode_e4m3(mids)
    lo = np.arange(126)
    expect = np.where(lo % 2 == 0, lo, lo + 1).astype(np.uint8)
    np.testing.assert_array_equal(got, expect)
    np.testing.assert_array_equal(oracle.encode_e4m3(np.float32([449.0, 1e30, -500.0])), [0x7E, 0x7E, 0xFE])
    assert oracle.encode_e4m3(np.float32([-0.0]))[0] == 0x80


def test_quantizer_matches_torch_cast(oracle):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((9, 7168)).astype(np.float32) * rng.choice([1e-6, 1e-2, 1.0, 300.0], (9, 1))
    x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    x[2] = 0.0                                  # all-zero token: scale 1, codes 0
    x[3, 128:256] = -0.0
    codes, scale = oracle.quantize_hidden(x)
    assert codes.shape == (9, 7168) and scale.shape == (56, 9)
    assert (scale[:, 2] == 1.0).all() and (codes[2] == 0).all()
    assert (codes[3, 128:256] == 0x80).all()
    y = x.reshape(9, 56, 128) / scale.T[:, :, None]
    ref = torch.from_numpy(y.astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(codes, ref.reshape(9, 7168))
    # amax of every nonzero block maps to the top code
    top = np.abs(oracle.decode_e4m3(codes).reshape(9, 56, 128)).max(axis=2)
    assert np.allclose(top[scale.T != 1.0], 448.0)
