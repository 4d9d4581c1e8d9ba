"""Multi-GPU checks through torchrun (each skipped with fewer GPUs than ranks):
tensor-parallel prefill / decode logits and generations, pipeline, FLUX
sequence-parallel, expert-parallel and FSDP paths against their single-GPU
counterparts, at 2 ranks and (where the box has them) 4 and 8."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _torchrun(module, n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={29500 + os.getpid() % 400}",
           "-m", module]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    return r.stdout


def test_pipeline_parallel_two_stages():
    out = _torchrun("rlx_models_b200.parallel.pp_check", 2)
    assert '"match": true' in out


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tensor_parallel(n):
    out = _torchrun("rlx_models_b200.parallel.tp_check", n)
    assert '"ok_all_ranks": false' not in out and out.count('"ok_all_ranks": true') == 4


def test_flux_sequence_parallel_two_ranks():
    out = _torchrun("rlx_models_b200.parallel.flux_sp_check", 2)
    assert '"ok": true' in out


def test_expert_parallel_fused_combine_two_ranks():
    out = _torchrun("rlx_models_b200.parallel.ep_check", 2)
    assert '"ok_all_ranks": false' not in out and out.count('"ok_all_ranks": true') == 2


def test_fsdp_push_reduce_scatter_two_ranks():
    out = _torchrun("rlx_models_b200.train.fsdp_check", 2)
    assert '"ok_all_ranks": true' in out
