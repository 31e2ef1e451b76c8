"""Host-side pieces that need no GPU: the scratch layouts the Python helpers
describe agree with the library's own size functions, the MoE scratch layout
is ordered and aligned, and the oracle's MoE routing/permutation and integer
weight quantization follow their definitions (checked against plain loops)."""
import numpy as np
import pytest

import mpp41
import oracle as O

up = lambda n: (n + 255) & ~255


@pytest.mark.parametrize("T,H,I", [(1, 512, 1024), (128, 1024, 4096), (77, 4096, 14336)])
def test_scratch_layouts_match_the_library(T, H, I):
    o = mpp41.w4a4_scratch_layout(T, H, I)
    assert mpp41.w4a4_scratch_bytes(T, H, I) == o[3] + up(T * I // 32)
    o = mpp41.nvfp4_scratch_layout(T, H, I)
    assert mpp41.nvfp4_scratch_bytes(T, H, I) == o[5] + up(8)
    o = mpp41.w8a8_scratch_layout(T, H, I)
    assert mpp41.w8a8_scratch_bytes(T, H, I) == o[4] + up(T * 4)
    assert all(v % 256 == 0 for v in o)


@pytest.mark.parametrize("shared", [0, 2048])
def test_moe_scratch_layout(shared):
    d = mpp41.moe_desc(512, 7168, 2048, 32, 8, shared)
    total, off = mpp41.moe_scratch_layout(d)
    vals = [off[k] for k in mpp41.MOE_PARTS]
    assert vals == sorted(vals) and all(v % 256 == 0 for v in vals)
    R = 512 * 8
    assert off["y"] - off["ms"] >= R * 2048 // 32
    assert total - off["sy"] == (up(512 * 7168 * 4) if shared else 0)
    ep = mpp41.moe_ep_scratch_bytes(d, 8, 8 * R)
    assert ep > total
    assert mpp41.moe_ep_scratch_bytes(d, 3, R) == 0      # experts must divide over the ranks


def test_oracle_routing_against_loops():
    rng = np.random.default_rng(4)
    logits = rng.integers(-3, 4, (50, 32)).astype(np.float32)   # many exact ties
    ids, w = O.moe_route(logits, 6)
    for t in range(50):
        order = sorted(range(32), key=lambda e: (-logits[t, e], e))[:6]
        assert list(ids[t]) == order
        e = np.exp(logits[t, order].astype(np.float64) - logits[t, order[0]])
        assert np.allclose(w[t], e / e.sum())
    perm, counts = O.moe_permutation(ids, 32)
    expect = [a for e in range(32) for a in range(ids.size) if ids.reshape(-1)[a] == e]
    assert list(perm) == expect and counts.sum() == ids.size


@pytest.mark.parametrize("bits", [8, 4, 2])
def test_oracle_int_rows_against_loops(bits):
    rng = np.random.default_rng(bits)
    w = rng.standard_normal((5, 64)).astype(np.float32)
    w[2] = 0
    packed, scales = O.quantize_int_rows(w, bits)
    qmax = {8: 127, 4: 7, 2: 1}[bits]
    per = 8 // bits
    for r in range(5):
        amax = np.float32(np.abs(w[r]).max())
        s = np.float32(amax / np.float32(qmax)) if amax > 0 else np.float32(1)
        assert scales[r] == s
        for k in range(64):
            q = int(np.clip(np.rint(w[r, k] / s), -qmax, qmax))
            byte = packed[r, k // per]
            got = (int(byte) >> (bits * (k % per))) & ((1 << bits) - 1)
            assert got == (q & ((1 << bits) - 1))
