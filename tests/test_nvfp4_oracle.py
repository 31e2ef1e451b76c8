"""CPU checks of the NVFP4 restatement: the recipe's invariants (the block
holding the tensor maximum gets scale code 0x7E = 448, every element decodes
within half an E2M1 step of the input, all-zero blocks stay zero) and a
decode of hand-built bytes."""
import numpy as np

import oracle as O


def test_nvfp4_recipe_invariants():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 256)) * 0.05).astype(np.float32)
    w[5, 32:48] = 0
    pk, sc, ts = O.quantize_nvfp4(w)
    amax = np.abs(w).max()
    assert ts == np.float32(amax / np.float32(2688))
    r, c = np.unravel_index(np.abs(w).argmax(), w.shape)
    assert sc[r, c // 16] == 0x7E
    d = O.decode_nvfp4(pk, sc, ts, 64, 256)
    assert np.all(d[5, 32:48] == 0)
    scale = np.repeat(np.array([O.lib().orc_e4m3_decode(int(v)) for v in sc.ravel()]).reshape(sc.shape), 16, 1) * ts
    step = np.where(np.abs(w) / np.maximum(scale, 1e-30) >= 4, 2.0, np.where(np.abs(w) / np.maximum(scale, 1e-30) >= 2, 1.0, 0.5))
    assert np.all(np.abs(d - w) <= 0.5 * step * scale + 1e-12)


def test_nvfp4_decode_known_bytes():
    packed = np.array([[0x71, 0xF9]], np.uint8)      # nibbles 1, 7, 9, 15 -> 0.5, 6, -0.5, -6
    scales = np.array([[0x38]], np.uint8)            # UE4M3 0x38 = 1.0
    d = O.decode_nvfp4(np.pad(packed, ((0, 0), (0, 6))), scales, 0.25, 1, 16)
    assert list(d[0, :4]) == [0.125, 1.5, -0.125, -1.5]
