"""Pipeline-parallel correctness check (launch with torchrun on N GPUs).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m rlx_models_b200.parallel.pp_check

Builds the same seeded decoder split over N pipeline stages and, on rank 0,
an unsplit copy; greedy generations of a few prompts through the engine must
agree (first tokens equal, mean common-prefix fraction >= 0.6: the split-K
decode GEMMs sum with atomics, so bits can differ between runs and a tiny
random model's greedy continuation may part at a near-tie).
Prints one JSON line from rank 0 and exits non-zero on a mismatch.
"""
from __future__ import annotations

import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    from rlx_models_b200 import config as C
    from rlx_models_b200 import ops
    from rlx_models_b200.models.decoder import DecoderLM
    from rlx_models_b200.parallel.pipeline import PipelineDecoderLM
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from rlx_models_b200.weights.init import random_weights

    cfg = C.tiny(num_hidden_layers=5, hidden_size=1024, intermediate_size=2048, num_attention_heads=8,
                 num_key_value_heads=4, head_dim=128, vocab_size=4096)
    w = random_weights(cfg, seed=5, device=dev)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 300, 64, 17)]
    sp = SamplingParams(max_new_tokens=24, ignore_eos=True)
    ecfg = EngineConfig(max_num_seqs=8, max_model_len=512, num_blocks=256, max_batched_tokens=256)
    pp = PipelineDecoderLM(cfg, w, device=dev, pp_rank=rank, pp_size=world)
    out_pp = [o.token_ids for o in LLMEngine(pp, ecfg).generate(prompts, sp)]
    ops.check_errors(dev)
    ok = True
    res = {"world": world, "layers_per_stage": [list(pp.layer_range)]}
    if rank == 0:
        ref = DecoderLM(cfg, w, device=dev)
        out_ref = [o.token_ids for o in LLMEngine(ref, ecfg).generate(prompts, sp)]
        def prefix(a, b):
            n = 0
            while n < min(len(a), len(b)) and a[n] == b[n]:
                n += 1
            return n / max(1, len(b))
        first = all(a[0] == b[0] for a, b in zip(out_pp, out_ref))
        agree = sum(prefix(a, b) for a, b in zip(out_pp, out_ref)) / len(out_ref)
        ok = first and agree >= 0.6
        res.update(match=ok, exact=out_pp == out_ref, prefix_agreement=round(agree, 3),
                   tokens=sum(len(o) for o in out_pp))
        print(json.dumps(res), flush=True)
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
