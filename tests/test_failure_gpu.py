"""Device-side failure path without a GPU fault: a bounded wait on a flag
that nothing sets runs out (~2 s), records its code in the status word and
returns; the host raises KernelError and the context stays usable."""
import pytest
import torch

from rlx_models_b200 import ops
from rlx_models_b200.ops._ext import KernelError, ext, scratch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives(cuda):
    st = scratch(cuda).status
    ops.check_errors(cuda)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    ok = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    ext().flag_wait_probe(flag, 1, st, ok)  # nothing will ever set the flag
    torch.cuda.synchronize()
    assert int(ok) == 0
    with pytest.raises(KernelError) as e:
        ops.check_errors(cuda)
    assert e.value.code == 5 and e.value.detail == 9
    # the status word was cleared and the device keeps working
    flag.fill_(7)
    ext().flag_wait_probe(flag, 1, st, ok)
    x = torch.randn(64, 256, device=cuda).bfloat16()
    w = torch.randn(384, 256, device=cuda).bfloat16()
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    assert int(ok) == 1
    ops.check_errors(cuda)
    assert torch.allclose(y.float(), x.float() @ w.float().T, rtol=2e-2, atol=2e-1)
