"""Whole model expert parallel, one rank per GPU (run by tests/test_gpu_model.py through torchrun):

    torchrun --nproc-per-node G --master-addr 127.0.0.1 --master-port P tests/model_ep_check.py

Every rank builds the same small random-init Qwen2-MoE model (fp32), feeds its own token ids and
swaps every MoE block with replace_qosmoe_layer at world_size G (process_group set, contiguous
expert placement, harmony on).  Its logits must equal, on every rank, those of the same model
swapped at world_size 1 (the expert-parallel block output is bit-identical to the one-GPU block)
and stay within 1e-4 of the unswapped transformers model."""
import copy
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from hf_models import QWEN_PLUGIN, qwen_model, token_batch  # noqa: E402
from dsca_moe_b200 import QoSMoEConfig, RequestStateTable, get_qosmoe_layers, replace_qosmoe_layer  # noqa: E402


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-300))


def swap(model, rank, world, group, B, S):
    cfg = QoSMoEConfig(rank=rank, world_size=world, expert_cache_size=1 << 10, process_group=group)
    replace_qosmoe_layer(model, config=cfg, **QWEN_PLUGIN)
    layers = get_qosmoe_layers(model)
    ctx = RequestStateTable(cfg).build_context({"attention_mask": torch.ones(B, S, dtype=torch.long)})
    for layer in layers:
        layer.set_runtime_context(ctx)
    return layers


@torch.no_grad()
def main():
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    group = dist.group.WORLD
    B, S = 4, 64
    base = qwen_model(seed=7, layers=3).to(dev)
    ids = token_batch(base.config.vocab_size, B, S, seed=30 + rank).to(dev)
    ref = base(input_ids=ids).logits
    one = copy.deepcopy(base)
    swap(one, 0, 1, None, B, S)
    want = one(input_ids=ids).logits
    ep_layers = swap(base, rank, world, group, B, S)
    results = []
    for it in range(2):
        got = base(input_ids=ids).logits
        torch.cuda.synchronize()
        for layer in ep_layers:
            layer.engine.check()
        results.append({"rank": rank, "iter": it, "equal_to_1gpu": bool(torch.equal(got, want)),
                        "max_rel_err_vs_1gpu": rel(got, want), "max_rel_err_vs_transformers": rel(got, ref)})
    ok = all(r["max_rel_err_vs_1gpu"] < 1e-6 and r["max_rel_err_vs_transformers"] < 1e-4 for r in results)
    for layer in ep_layers:
        layer.engine.close()
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    gathered = [None] * world
    dist.all_gather_object(gathered, results)
    if rank == 0:
        print(json.dumps({"world": world, "ok": bool(flag.item()), "results": sum(gathered, [])}))
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
