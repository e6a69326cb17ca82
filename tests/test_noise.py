"""The render's start image (src/u15-generator.cc:394-417) and its noise
scale (GenConfig::init_noise_scale, src/u15-config.cc:106-122), on the host.

The reference draws the image with std::mt19937_64(seed) and
std::normal_distribution<float>(0, 1), scaled in double by the noise scale.
u15c_init_noise is checked bit for bit against the CPU checker's draw
(oracle/u15_noise.cc, the same library types), the engine against the C++
standard's known answer, and the noise scale against the values the
reference's own config test expects (tests/u15-config-test.cc:136-141)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from u15b200 import _lib as L


def draw(seed, scale, n):
    out = np.empty(n, np.float32)
    assert L.lib().u15c_init_noise(seed, scale, C.c_void_p(out.ctypes.data), n) == 0
    return out


def scale_of(tokens, mode=L.NOISE_RESOLUTION, s=1.0, mx=16.0, base=64):
    out = C.c_double()
    assert L.lib().u15c_init_noise_scale(tokens, mode, s, mx, base, C.byref(out)) == 0
    return out.value


def test_engine_known_answer():
    # [rand.predef]: the 10000th consecutive invocation of a default-constructed
    # mt19937_64 (seed 5489) produces 9981545732273789042
    assert O.mt19937_64_nth(5489, 10000) == 9981545732273789042


@pytest.mark.parametrize("seed,scale,n", [(0, 1.0, 3 * 32 * 32), (42, 4.0, 3 * 64 * 48 + 1),
                                          (2 ** 63 + 5, 8.0, 12345), (7, 16.0, 1)])
def test_draw_bit_identical(seed, scale, n):
    got = draw(seed, scale, n)
    want = O.init_noise(seed, scale, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_draw_statistics_and_seed():
    a = draw(1, 4.0, 3 * 256 * 256)
    assert abs(a.mean()) < 0.05 and abs(a.std() - 4.0) < 0.05
    assert not np.array_equal(draw(2, 4.0, 64), draw(1, 4.0, 64))
    # the draw order is the image's: a prefix of a longer draw is the shorter draw
    assert np.array_equal(draw(3, 1.0, 1000)[:999], draw(3, 1.0, 999))


def test_noise_scale_reference_values():
    # the reference's own expectations (tests/u15-config-test.cc:136-141)
    assert scale_of(64) == pytest.approx(1.0)
    assert scale_of(256) == pytest.approx(2.0)
    assert scale_of(1024) == pytest.approx(4.0)
    assert scale_of(1 << 20) == pytest.approx(16.0)
    assert scale_of(1 << 20) <= 16.0
    # the other branches of the rule, against the checker
    for tokens in (1, 64, 1000, 4096, 40000):
        for mode in (L.NOISE_CONSTANT, L.NOISE_RESOLUTION, L.NOISE_DYNAMIC_SQRT):
            for s, mx, base in ((1.0, 16.0, 64), (0.5, 3.0, 256), (2.0, 100.0, 0)):
                assert scale_of(tokens, mode, s, mx, base) == \
                    O.init_noise_scale(tokens, mode, s, mx, base)
    assert scale_of(4096, L.NOISE_DYNAMIC_SQRT) == pytest.approx(np.sqrt(8.0))
    assert scale_of(4096, L.NOISE_CONSTANT, 3.0) == 3.0


def test_refusals():
    out = C.c_double()
    assert L.lib().u15c_init_noise_scale(64, 7, 1.0, 16.0, 64, C.byref(out)) == L.EINVAL
    assert L.lib().u15c_init_noise(0, 1.0, None, 4) == L.EINVAL
