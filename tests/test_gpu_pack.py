"""K2, the activation pack, through the C ABI, against the oracle: the bfp16
bytes must be identical and the bf16 copy must be the exact decoded values."""
import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O
from gpu_util import dev, host, bf16_bits_of

pytestmark = pytest.mark.gpu


def check_pack(x: np.ndarray, m_pad=None):
    T, K = x.shape
    m_pad = m_pad or Z.pad_to(max(T, 1), 128)
    ab, ah = Z.pack_activations(dev(x), m_pad)
    full = np.zeros((m_pad, K), np.float32)
    full[:T] = x
    want = O.pack_a(full)
    got = host(ab)
    assert np.array_equal(got, want), f"bytes differ at {np.flatnonzero(got != want)[:8]}"
    dec = O.decode_blocks(O.encode_blocks(full)).reshape(m_pad, K)
    assert np.array_equal(host(ah).view(np.uint16), bf16_bits_of(dec))


def test_pack_golden_256x128():
    g = np.load(Z.PKG_DIR.parent / "tests" / "golden" / "pack_a_256x128.npz")
    ab, _ = Z.pack_activations(dev(g["x"]))
    assert np.array_equal(host(ab), g["bytes"])


@pytest.mark.parametrize("T,K", [(128, 64), (256, 384), (1024, 2560), (1000, 512), (1, 64), (130, 4096)])
def test_pack_adversarial(T, K):
    check_pack(O.make_data(T * K, T + K).reshape(T, K))


def test_pack_normal_with_outliers():
    check_pack(O.activations(2048, 2048, 1, outliers=True))


def test_pack_specials():
    g = np.load(Z.PKG_DIR.parent / "tests" / "golden" / "codec.npz")
    x = g["x"][-56:]
    x = np.concatenate([x, np.zeros(64 - 56, np.float32)]).reshape(1, 64)
    ab, ah = Z.pack_activations(dev(np.repeat(x, 16, axis=0)))
    got = host(ab)
    want = O.pack_a(np.concatenate([np.repeat(x, 16, axis=0), np.zeros((112, 64), np.float32)]))
    assert np.array_equal(got, want)


def test_pack_only_bf16_and_only_bytes():
    x = O.activations(384, 1024, 3)
    ab, _ = Z.pack_activations(dev(x), want_bf16=False)
    _, ah = Z.pack_activations(dev(x), want_bytes=False)
    assert np.array_equal(host(ab), O.pack_a(x))
    assert np.array_equal(host(ah).view(np.uint16), bf16_bits_of(O.decode_blocks(O.encode_blocks(x)).reshape(384, 1024)))


def test_pack_full_size_slices():
    # config 2's activation shape, 8192 x 2560: every 128-row block is a
    # self-contained run of tiles, so sampled blocks are checked exactly
    K = 2560
    x = torch.randn(8192, K, device="cuda", generator=torch.Generator("cuda").manual_seed(7))
    ab, ah = Z.pack_activations(x)
    hb, hh = host(ab), host(ah).view(np.uint16)
    run = 128 * K * 9 // 8
    for r0 in (0, 2048, 4096, 8064):
        xs = host(x[r0:r0 + 128])
        assert np.array_equal(hb[r0 // 128 * run:(r0 // 128 + 1) * run], O.pack_a(xs)), r0
        assert np.array_equal(hh[r0:r0 + 128], bf16_bits_of(O.decode_blocks(O.encode_blocks(xs)).reshape(128, K)))
    # the bf16 copy and the bytes agree everywhere: summed decoded values per 128-row block
    dec = (ah.to(torch.int32) << 16).view(torch.float32)
    assert torch.isfinite(dec).all()
