"""Checkpoint reading on the CPU: the safetensors container, the affine-pack
shape rule of bind_matrix_ (src/u15-weights.cc:248-325), and the reference
fixture's packing restated (tests/u15-m5-test.cc:263-310)."""
import numpy as np
import pytest

from ckpt_util import bf16_bits, dequant, from_bf16_bits, quantize


def test_safetensors_round_trip(tmp_path):
    from u15b200.checkpoint import SafeTensors, write_safetensors
    rng = np.random.default_rng(1)
    t = {"a.f32": rng.normal(size=(3, 5)).astype(np.float32),
         "b.f16": rng.normal(size=(7,)).astype(np.float16),
         "c.u32": rng.integers(0, 2**32, (4, 2), dtype=np.uint64).astype(np.uint32),
         "d.bf16": ("BF16", bf16_bits(rng.normal(size=(2, 3)).astype(np.float32)))}
    write_safetensors(str(tmp_path / "m.safetensors"), t)
    st = SafeTensors(str(tmp_path))
    for k, v in t.items():
        want = v[1] if isinstance(v, tuple) else v
        assert np.array_equal(st.array(k), want) and st.shape(k) == want.shape
    assert st.dtype("d.bf16") == "BF16" and "missing" not in st


def test_pack_shape_rule():
    from u15b200.checkpoint import pack_shape
    K = 4096
    assert pack_shape(K, K // 64, K * 8 // 32) == (8, 64)
    assert pack_shape(K, K // 32, K * 4 // 32) == (4, 32)
    assert pack_shape(K, K // 16, K * 8 // 32) is None      # group 16: not a pack this reads
    assert pack_shape(K, K // 64, K * 2 // 32) is None      # 2-bit
    assert pack_shape(K, K // 64 + 1, K * 8 // 32) is None  # does not close
    assert pack_shape(12288, 12288 // 64, 12288 * 8 // 32) == (8, 64)


@pytest.mark.parametrize("bits,group,sdt", [(8, 64, "BF16"), (8, 32, "F16"), (4, 64, "F16")])
def test_fixture_packing_restated(bits, group, sdt):
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, (16, 256)).astype(np.float32)
    codes, s, b, c = quantize(w, group, bits, sdt)
    per = 32 // bits
    # the codes unpack to the quantized levels, little end first
    for k in range(per):
        assert np.array_equal((codes >> np.uint32(k * bits)) & np.uint32((1 << bits) - 1),
                              c.reshape(16, -1, per)[:, :, k])
    deq = dequant(c, s, b, group, sdt)
    step = np.repeat(from_bf16_bits(s) if sdt == "BF16" else s.astype(np.float32), group, 1)
    # within one level: half a level of rounding, plus up to half a level at
    # the top of a group where the bf16-rounded scale falls short of the
    # range (the fixture rounds the scale before choosing codes); plus the
    # bf16 rounding of the value
    assert (np.abs(deq - w) <= 1.01 * np.abs(step) + 2 ** -8 * np.abs(w) + 1e-7).all()
    assert np.median(np.abs(deq - w) / np.abs(step)) < 0.3
