"""Expert-parallel parity check, one rank per GPU (run by tests/test_gpu_ep.py through torchrun):

    torchrun --nproc-per-node G --master-addr 127.0.0.1 --master-port P tests/ep_check.py

Each rank routes its own tokens, the harmony plan moves hot-expert tokens between GPUs, and the
block's output on every rank must equal the single-GPU result of the same tokens: routing
bit-exact, outputs within 2e-2 (they come out bit-identical when the plan does not matter to the
row arithmetic, and the check reports that).  Covers the Qwen top-4 + shared block (even and
uneven placements, harmony on and off) and the Switch top-1 block (whose multi-GPU output the
reference leaves uncombined, src/harmonymoe/scheduler.py:158-175)."""
import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from dsca_moe_b200 import _lib as L  # noqa: E402
from dsca_moe_b200 import synthetic as syn  # noqa: E402
from dsca_moe_b200.engine import MoEEngine, pack_relu, pack_swiglu, plan_harmony  # noqa: E402


def rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def case_qwen(rank, world, dev, group, e2g, eq_tokens, exchange, T=512):
    d, E, I, Is = 1024, 60, 256, 512
    Wg, _ = syn.router_weight(E, d, 71, zipf_s=1.5, dtype="bf16")
    g = torch.Generator(device=dev)
    g.manual_seed(72)

    def n(*s):
        return (torch.randn(*s, generator=g, device=dev) * 0.03).to(torch.bfloat16)

    w = dict(gate=n(E, I, d), up=n(E, I, d), down=n(E, d, I), sg=n(Is, d), su=n(Is, d), sd=n(d, Is), g=n(d))
    pe = pack_swiglu(w["gate"], w["up"], w["down"], shared=(w["sg"], w["su"], w["sd"]), device=dev)
    Wt = torch.from_numpy(Wg).to(dev, torch.bfloat16)
    ep = MoEEngine(Wt, pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK, shared_gate_weight=w["g"], rank=rank,
                   world=world, group=group, expert_to_gpu=e2g, eq_tokens=eq_tokens, exchange=exchange)
    one = MoEEngine(Wt, pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK, shared_gate_weight=w["g"])
    x = torch.from_numpy(syn.hidden_states(T, d, 700 + rank, "bf16")).to(dev, torch.bfloat16)
    return ep, one, x


def case_switch(rank, world, dev, group, e2g, eq_tokens, exchange, T=640):
    d, E, F = 768, 64, 1024
    Wr, _ = syn.router_weight(E, d, 81, zipf_s=1.0, dtype="bf16")
    g = torch.Generator(device=dev)
    g.manual_seed(82)
    wi = (torch.randn(E, F, d, generator=g, device=dev) * 0.03).to(torch.bfloat16)
    wo = (torch.randn(E, d, F, generator=g, device=dev) * 0.03).to(torch.bfloat16)
    pe = pack_relu(wi, wo, device=dev)
    Wt = torch.from_numpy(Wr).to(dev, torch.bfloat16)
    ep = MoEEngine(Wt, pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1, rank=rank, world=world, group=group,
                   expert_to_gpu=e2g, eq_tokens=eq_tokens, exchange=exchange)
    one = MoEEngine(Wt, pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1)
    x = torch.from_numpy(syn.hidden_states(T, d, 800 + rank, "bf16")).to(dev, torch.bfloat16)
    return ep, one, x


def case_qwen_cache(rank, world, dev, group, e2g, eq_tokens, exchange, T=512):
    """The Qwen case with an expert cache of 8 device slots per rank (the reference's
    expert_cache_size < num_experts on every rank): experts are loaded into slots per the QoS
    plan, and the output still equals the one-GPU result."""
    ep, one, x = case_qwen(rank, world, dev, group, e2g, eq_tokens, exchange, T)
    cached = MoEEngine(ep.router_weight, ep.experts, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                       shared_gate_weight=ep.shared_gate_weight, rank=rank, world=world, group=group,
                       expert_to_gpu=e2g, eq_tokens=eq_tokens, exchange=exchange, cache_slots=8)
    return cached, one, x


def case_qwen_fp8(rank, world, dev, group, e2g, eq_tokens, exchange, T=512):
    """The Qwen case with fp8-e4m3 expert weights (per-channel scales): the dispatch stores f16
    rows, the return kernel brings the bf16 outputs back; equal to the one-GPU fp8 result."""
    from dsca_moe_b200.engine import quantize_fp8

    ep, one, x = case_qwen(rank, world, dev, group, e2g, eq_tokens, exchange, T)
    pe8 = quantize_fp8(ep.experts)
    ep8 = MoEEngine(ep.router_weight, pe8, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                    shared_gate_weight=ep.shared_gate_weight, rank=rank, world=world, group=group,
                    expert_to_gpu=e2g, eq_tokens=eq_tokens, exchange=exchange)
    one8 = MoEEngine(ep.router_weight, pe8, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                     shared_gate_weight=ep.shared_gate_weight)
    return ep8, one8, x


def main():
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    group = dist.group.WORLD
    results = []
    uneven60 = np.array([min(world - 1, (e * world * world) // (60 * (world + 1))) for e in range(60)], np.int32)
    cases = []
    for exchange in ("p2p", "p2p-fused", "p2p-graph", "nccl"):
        cases += [
            (f"qwen contiguous, harmony, {exchange}", case_qwen, None, 150, exchange),
            (f"qwen contiguous, fixed, {exchange}", case_qwen, None, -1, exchange),
            (f"qwen uneven placement, harmony, {exchange}", case_qwen, uneven60, 150, exchange),
            (f"switch top-1, harmony, {exchange}", case_switch, None, 150, exchange),
        ]
    cases.append(("qwen contiguous, harmony, p2p, expert cache 8 slots", case_qwen_cache, None, 150, "p2p"))
    cases.append(("qwen contiguous, harmony, p2p, fp8-e4m3 weights", case_qwen_fp8, None, 150, "p2p"))
    cases.append(("qwen contiguous, harmony, p2p, QoS scores on the main stream", case_qwen, None, 150, "p2p-qosmain"))
    cases.append(("qwen contiguous, harmony, p2p, QoS scores and priority exchange on their own stream", case_qwen,
                  None, 150, "p2p-qospar"))
    ok = True
    for name, fn, e2g, eq, exchange in cases:
        ep, one, x = fn(rank, world, dev, group, e2g, eq, "nccl" if exchange == "nccl" else "p2p")
        ep.ep_return = "fused" if exchange == "p2p-fused" else "overlap"
        if exchange == "p2p-qosmain":
            ep.qos_stream = "main"
        if exchange == "p2p-qospar":
            ep.qos_stream = "parallel"
        graph = None
        if exchange == "p2p-graph":
            # the forward captured once (collective), replayed on new contents of its input buffer
            xbuf = x.clone()
            graph = ep.capture(xbuf)
        for it in range(3):
            if graph is not None:
                x = torch.from_numpy(syn.hidden_states(x.shape[0], x.shape[1], 900 + 10 * it + rank, "bf16")).to(
                    dev, torch.bfloat16)
                xbuf.copy_(x)
                graph.replay()
                r_ep = graph.result
            else:
                r_ep = ep.forward(x)
            r_one = one.forward(x)
            torch.cuda.synchronize()
            ep.check()
            one.check()
            same_route = torch.equal(r_ep["topk_ids"], r_one["topk_ids"]) and torch.equal(r_ep["logits"], r_one["logits"])
            if exchange in ("p2p", "p2p-qosmain", "p2p-qospar") and ep.qos_order:
                # the QoS order is the summed priorities' order, the same on every rank
                order, prio = ep.read_qos_order()
                mine = torch.from_numpy(prio.copy()).to(dev)
                allp = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(allp, mine)
                same_route = same_route and all(torch.equal(allp[0], t) for t in allp)
                same_route = same_route and order.tolist() == sorted(range(ep.E), key=lambda e: (-float(prio[e]), e))
            err = rel(r_ep["out"], r_one["out"])
            exact = torch.equal(r_ep["out"], r_one["out"])
            S, _ = ep.read_plan()
            migrated = int(S.sum() - sum(S[:, e, ep.expert_to_gpu[e]].sum() for e in range(S.shape[1])))
            # the plan the devices computed equals the host planner's on the all-gathered counts
            meta = torch.empty(world, ep.E, dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(meta, r_one["counts"].contiguous())
            plan_ok = bool(np.array_equal(S, plan_harmony(meta.cpu().numpy(), ep.expert_to_gpu, eq)))
            good = same_route and plan_ok and err < 2e-2 and torch.isfinite(r_ep["out"].float()).all().item()
            ok &= bool(good)
            results.append({"case": name, "iter": it, "rank": rank, "routing_equal": bool(same_route),
                            "plan_equal": plan_ok, "max_rel_err": err, "bit_identical": bool(exact),
                            "tokens_migrated": migrated})
        del graph
        ep.close()
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
