"""GPU: the producer-side activation quantiser equals the oracle bit for bit
(e4m3 bytes and fp32 scales), for f32 and bf16 inputs, and feeds the operator."""
import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T", [1, 7, 300])
def test_quantize_bit_exact(T, dtype, pkg, oracle):
    g = torch.Generator().manual_seed(T)
    x = (torch.randn(T, 7168, generator=g) * 2.5).to(dtype)
    x[0, 128:256] = 0
    q, s = pkg.quantize_activations(x.cuda())
    q_ref, s_ref = oracle.quantize_rows(x.float().numpy())
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), q_ref)


def test_quantized_activations_feed_the_operator(pkg, oracle):
    x = pkg.inputs.make_inputs(24, seed=77, device="cuda", weight_experts=4)
    g = torch.Generator(device="cuda").manual_seed(5)
    act = torch.randn(24, 7168, generator=g, device="cuda").to(torch.bfloat16)
    hq, hs = pkg.quantize_activations(act)
    args = list(x.args())
    args[2], args[3] = hq, hs
    out = pkg.run(*args)
    assert_close(out.float().cpu().numpy(), oracle.moe_forward(*args), what="quantised activations")
