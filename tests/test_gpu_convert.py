"""K1, the weight conversion, through the C ABI, against the oracle: for
each GGUF type, bytes identical to pack_b(to_float(raw)) and the bf16 copy
the exact decoded values; fused gate/up and N-shards too."""
import numpy as np
import pytest

import zest_b200 as Z
from oracle import oracle as O
from gpu_util import dev, host, bf16_bits_of

pytestmark = pytest.mark.gpu

TYPES = [O.F32, O.F16, O.Q8_0, O.Q4_K, O.Q6_K, O.IQ3_S]


@pytest.fixture(scope="module", autouse=True)
def grid():
    Z.load_iq3s_grid()


def want_b(values: np.ndarray, n_pad: int):
    N, K = values.shape
    full = np.zeros((n_pad, K), np.float32)
    full[:N] = values
    return O.pack_b(full), bf16_bits_of(O.decode_blocks(O.encode_blocks(full)).reshape(n_pad, K))


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("N,K", [(512, 256), (1000, 512), (64, 1024)])
def test_convert(qt, N, K):
    raw = O.quantize(qt, O.weights_f32(N, K, qt * 100 + N))
    bb, bh = Z.convert_weight(qt, dev(raw), N, K)
    wb, wh = want_b(O.dequant(qt, raw, N, K), Z.pad_to(N, 512))
    assert np.array_equal(host(bb), wb)
    assert np.array_equal(host(bh).view(np.uint16), wh)


def test_convert_q8_0_narrow_k():
    # K % 256 != 0 takes the 64-wide path
    qt, N, K = O.Q8_0, 512, 320
    raw = O.quantize(qt, O.weights_f32(N, K, 5))
    bb, bh = Z.convert_weight(qt, dev(raw), N, K)
    wb, wh = want_b(O.dequant(qt, raw, N, K), 512)
    assert np.array_equal(host(bb), wb) and np.array_equal(host(bh).view(np.uint16), wh)


def test_convert_golden_pack_b():
    g = np.load(Z.PKG_DIR.parent / "tests" / "golden" / "pack_b_512x128.npz")
    bb, _ = Z.convert_weight(O.F32, dev(g["w"].view(np.uint8)), 512, 128)
    assert np.array_equal(host(bb), g["bytes"])


@pytest.mark.parametrize("name,qt", [("q8_0", O.Q8_0), ("q4_k", O.Q4_K), ("q6_k", O.Q6_K), ("iq3_s", O.IQ3_S)])
def test_convert_dequant_golden(name, qt):
    g = np.load(Z.PKG_DIR.parent / "tests" / "golden" / f"dequant_{name}.npz")
    _, bh = Z.convert_weight(qt, dev(g["raw"]), 16, 512)
    want = bf16_bits_of(O.decode_blocks(O.encode_blocks(g["values"])).reshape(16, 512))
    assert np.array_equal(host(bh)[:16].view(np.uint16), want)


def test_gate_up_golden():
    g = np.load(Z.PKG_DIR.parent / "tests" / "golden" / "gate_up_256x64.npz")
    bb, _ = Z.convert_gate_up(O.F32, dev(g["gate"].view(np.uint8)), dev(g["up"].view(np.uint8)), 256, 64)
    assert np.array_equal(host(bb), g["bytes"])


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K])
def test_gate_up_padded(qt):
    F, K = 300, 256  # F padded to 512 -> 1024 rows
    gr = O.quantize(qt, O.weights_f32(F, K, 1))
    ur = O.quantize(qt, O.weights_f32(F, K, 2))
    bb, bh = Z.convert_gate_up(qt, dev(gr), dev(ur), F, K)
    gp = np.zeros((512, K), np.float32)
    up = np.zeros((512, K), np.float32)
    gp[:F] = O.dequant(qt, gr, F, K)
    up[:F] = O.dequant(qt, ur, F, K)
    inter = O.interleave_gate_up(gp, up)
    assert np.array_equal(host(bb), O.pack_b(inter))
    assert np.array_equal(host(bh).view(np.uint16), bf16_bits_of(O.decode_blocks(O.encode_blocks(inter)).reshape(1024, K)))


def test_shard_rows():
    # rows [row0, row0 + n) of a weight, as one GPU of an N-sharded job converts them
    qt, N, K = O.Q4_K, 2048, 512
    raw = O.quantize(qt, O.weights_f32(N, K, 9))
    vals = O.dequant(qt, raw, N, K)
    for row0, n in ((0, 512), (512, 1024), (1536, 512)):
        bb, bh = Z.convert_weight(qt, dev(raw), N, K, row0=row0, n_rows=n)
        wb, wh = want_b(vals[row0:row0 + n], Z.pad_to(n, 512))
        assert np.array_equal(host(bb), wb) and np.array_equal(host(bh).view(np.uint16), wh)
