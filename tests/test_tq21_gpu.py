"""TQ2_1 blocks (the fork's static mixed-precision type, docs/RESULTS.md:1451-1466): each
128-element block is the reference's TQ3_0 block of elements 0..31 followed by its TQ2_0
blocks of 32..63, 64..95 and 96..127.  The oracle is that composition of the compiled
reference C (quantize_row_tq3_0_ref / quantize_row_tq2_0_ref and the dequantizers): bytes and
float32 outputs must be equal, for f32, f16 and bf16 inputs, with outlier channels, zero and
tie-prone sub-blocks."""
import numpy as np
import pytest
import torch

from leankv_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref_tq21(orc, x):
    """Reference bytes and reconstruction of TQ2_1 blocks of float32 x (flat, multiple of 128)."""
    sub = x.reshape(-1, 4, 32)
    b3 = orc.ref_quantize(3, sub[:, 0])                       # [n, 14]
    b2 = orc.ref_quantize(2, sub[:, 1:]).reshape(-1, 3, 10)   # [n, 3, 10]
    blocks = np.concatenate([b3, b2.reshape(-1, 30)], axis=1)
    y3 = orc.ref_dequantize(3, b3).reshape(-1, 32)
    y2 = orc.ref_dequantize(2, b2.reshape(-1, 10)).reshape(-1, 96)
    return blocks, np.concatenate([y3, y2], axis=1).reshape(-1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_tq21_matches_reference_composition(orc, dtype):
    g = torch.Generator().manual_seed(21)
    x = torch.randn(3000, 128, generator=g)
    x[:, :4] *= 20.0                      # outlier channels inside the TQ3 part
    x[5] = 0.0                            # all-zero block
    x[7, 32:64] = 0.0                     # one all-zero TQ2 sub-block
    x[9] = torch.linspace(-1, 1, 128)     # values on level boundaries after scaling
    x = x.to(dtype)
    blocks = ops.quantize_tq2_1(x.to(DEV))
    assert blocks.shape == (3000, 1, 44)
    xf = x.float().numpy().reshape(-1)    # the reference takes float32: bf16/f16 convert exactly
    ref_blocks, ref_y = _ref_tq21(orc, xf)
    got = blocks.cpu().numpy().reshape(-1, 44)
    assert np.array_equal(got, ref_blocks), f"{int((got != ref_blocks).any(axis=1).sum())} blocks differ"
    y = ops.dequantize_tq2_1(blocks).cpu().numpy().reshape(-1)
    assert np.array_equal(y, ref_y)


def test_tq21_random_bytes_dequantize(orc):
    """Arbitrary block bytes (any scale, any code) decode like the reference dequantizers."""
    rng = np.random.default_rng(5)
    raw = rng.integers(0, 256, size=(4096, 44), dtype=np.uint8)
    y = ops.dequantize_tq2_1(torch.from_numpy(raw).to(DEV)).cpu().numpy().reshape(-1)
    ref = np.concatenate([orc.ref_dequantize(3, raw[:, :14]).reshape(-1, 32),
                          orc.ref_dequantize(2, raw[:, 14:].reshape(-1, 10)).reshape(-1, 96)], axis=1).reshape(-1)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(y[fin], ref[fin])
