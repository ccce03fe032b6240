"""Deterministic combine (moe_fp8_set_deterministic): repeated calls give
bit-identical outputs, within the parity bar of the oracle, for decode- and
prefill-shaped calls (the mode always runs the tile kernels)."""
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture
def deterministic(pkg):
    old = pkg.set_deterministic(True)
    yield
    pkg.set_deterministic(old)


@pytest.mark.parametrize("T,skewed", [(64, False), (600, True)])
def test_repeated_calls_are_bit_identical(T, skewed, pkg, oracle, deterministic):
    x = pkg.inputs.make_inputs(T, seed=5, device="cuda", skewed=skewed)
    outs = [pkg.run(*x.args()).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert pkg.read_device_error() == 0
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    err = assert_close(outs[0].float().cpu().numpy(), oracle.moe_forward(*x.args()), what=f"deterministic T={T}")
    print(f"deterministic T={T}: max_abs_err={err:.3e}")
