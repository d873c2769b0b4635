"""The export merge (tq_lora_merge): a quantized linear plus its scaled LoRA
product, bit for bit against the oracle's restatement (the rank sum in f32,
i ascending, every product and sum rounded alone), in f32 and rounded once to
bf16; without a pair it is the dequantized weight in f32."""
from __future__ import annotations

import numpy as np
import pytest

from _util import dev_bf16, dev_u32, host_bf16

# (rows, cols, bits, group, rank): rows not a multiple of the kernel's four,
# every code width and group size, ranks 0/8/16 and an odd one.
CASES = [
    (64, 256, 4, 64, 8),
    (37, 512, 8, 32, 16),
    (130, 384, 4, 128, 3),
    (8, 64, 4, 32, 0),
    (4864, 896, 4, 64, 8),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "r{}_c{}_b{}_g{}_k{}".format(*c))
def test_merge_matches_the_oracle_bit_for_bit(cuda, oracle, case):
    import torch

    from torobi_b200 import ops

    rows, cols, bits, group, rank = case
    rng = np.random.default_rng(21)
    w = oracle.normal_bf16(rng, (rows, cols), 0.02)
    c, s, b = oracle.quantize(w, bits, group)
    a = rng.standard_normal((rank, cols)).astype(np.float32) * 0.1 if rank else None
    bb = rng.standard_normal((rows, rank)).astype(np.float32) * 0.01 if rank else None
    scale = 2.0 if rank else 1.0
    want = oracle.lora_merge(c, s, b, bits, group, a, bb, scale)
    ta = torch.from_numpy(a).to(cuda) if rank else None
    tb = torch.from_numpy(bb).to(cuda) if rank else None
    args = (dev_u32(c, cuda), dev_bf16(s, cuda), dev_bf16(b, cuda), group, bits)
    got = ops.lora_merge(*args, lora_a=ta, lora_b=tb, scale=scale).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    got16 = host_bf16(ops.lora_merge(*args, lora_a=ta, lora_b=tb, scale=scale,
                                     dtype=torch.bfloat16))
    assert np.array_equal(got16, oracle.bf16_from_f32(want))


@pytest.mark.gpu
def test_merge_without_a_pair_is_the_dequantized_weight(cuda, oracle):
    from torobi_b200 import ops

    rng = np.random.default_rng(22)
    w = oracle.weights_with_outliers(rng, (96, 1024))
    c, s, b = oracle.quantize(oracle.bf16_from_f32(w), 4, 64)
    got = ops.lora_merge(dev_u32(c, cuda), dev_bf16(s, cuda), dev_bf16(b, cuda), 64, 4)
    want = oracle.f32_from_bf16(oracle.dequantize(c, s, b, 4, 64))
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.gpu
def test_merge_rejects_bad_arguments(cuda):
    import torch

    from torobi_b200 import ops

    c = torch.zeros(8, 8, dtype=torch.uint32, device=cuda)
    s = torch.zeros(8, 1, dtype=torch.bfloat16, device=cuda)
    a = torch.zeros(8, 64, device=cuda)
    with pytest.raises(ValueError):
        ops.lora_merge(c, s, s, 64, 4, lora_a=a)
    with pytest.raises(ValueError):
        ops.lora_merge(c, s, s, 64, 4, lora_a=a, lora_b=torch.zeros(8, 4, device=cuda))
