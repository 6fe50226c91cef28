"""MoE-block forward engine: packed expert weights, workspace, and the kernel sequence.

One GPU:   router (+ fused scan) -> permute -> grouped FFN (routed + shared) -> combine, all on
           the caller's current stream with device-side counts (no host sync).
G GPUs:    (exchange="p2p", the default) router -> counts pushed to every peer and the harmony
           plan computed on the device -> rows stored straight into the owners' receive buffers
           over NVLink -> grouped FFN on the received rows (+ the shared expert on local tokens,
           overlapping the exchange on a side stream) -> rows stored back into the senders'
           return buffers -> combine; no host sync, so a forward can be captured as a CUDA
           graph (MoEEngine.capture).  exchange="nccl": counts all-gather -> host plan -> NCCL
           grouped send/recv of the chunks, kept as the library-collective baseline.

Reference hot path: QoSMoELayer.forward (src/qosmoe/moe_layer.py:271-459) and
ShardedQwenMoE.forward (qwen_ep_adapter/qwen_ep.py:44-97).  Every expert's weights are
resident on every GPU (B200 HBM holds a whole layer), so tokens that the harmony plan migrates
to a GPU that does not own their expert are served from local HBM: replication needs no copy
on the critical path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import numpy as np
import torch

from . import _lib as L
from .qos import ExpertCache, QoSInputs, build_exec_plan, match_token_length

__all__ = ["PackedExperts", "pack_swiglu", "pack_relu", "MoEEngine", "ForwardGraph", "HostPipeline", "plan_harmony",
           "plan_layout"]


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return ctypes.c_void_p(t)
    return ctypes.c_void_p(t.data_ptr())


class _DevPtr:
    """A raw device pointer seen as a torch tensor (zero copy, through __cuda_array_interface__)."""

    _TYPESTR = {torch.bfloat16: "<f2", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}

    def __init__(self, ptr: int, shape, dtype):
        # bf16 has no numpy type string: expose it as 2-byte float and reinterpret below
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": self._TYPESTR[dtype],
                                         "data": (ptr, False), "version": 3}

    @staticmethod
    def tensor(ptr: int, shape, dtype, device):
        t = torch.as_tensor(_DevPtr(ptr, shape, dtype), device=device)
        return t.view(dtype) if dtype == torch.bfloat16 else t


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ceil(a, b):
    return (a + b - 1) // b


def _dt(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return L.BF16
    if dtype == torch.float32:
        return L.F32
    raise ValueError(f"unsupported dtype {dtype}")


# ----------------------------------------------------------------------------- packing
@dataclass
class PackedExperts:
    """Expert weights in the kernel layout (include/dsca_b200.h, dsca_ffn_args)."""
    act: int
    d: int
    inter: int
    E: int
    w1: torch.Tensor      # [E, n1p, d]
    w2: torch.Tensor      # [E, dp, ip]
    n1p: int
    ip: int
    dp: int
    # shared expert (SwiGLU, E = 1) or None
    ws1: torch.Tensor | None = None
    ws2: torch.Tensor | None = None
    s_inter: int = 0
    s_n1p: int = 0
    s_ip: int = 0
    # fp8-e4m3 weights: per packed-row (output channel) fp32 scales, weights = q * scale
    w1_scale: torch.Tensor | None = None
    w2_scale: torch.Tensor | None = None
    ws1_scale: torch.Tensor | None = None
    ws2_scale: torch.Tensor | None = None

    @property
    def fp8(self) -> bool:
        return self.w1.dtype == torch.float8_e4m3fn

    @property
    def dtype(self):
        """Activation dtype of the block (bf16 for fp8 weights)."""
        return torch.bfloat16 if self.fp8 else self.w1.dtype


def _quant_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row (output channel) e4m3 quantisation: scale = amax / 448, q = rne_e4m3(w / scale)."""
    wf = w.float()
    amax = wf.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (wf / scale).to(torch.float8_e4m3fn)
    return q.contiguous(), scale.squeeze(-1).contiguous()


def quantize_fp8(pe: PackedExperts) -> PackedExperts:
    """fp8-e4m3 copy of packed expert weights with per-output-channel fp32 scales."""
    w1, s1 = _quant_rows(pe.w1)
    w2, s2 = _quant_rows(pe.w2)
    out = PackedExperts(act=pe.act, d=pe.d, inter=pe.inter, E=pe.E, w1=w1, w2=w2, n1p=pe.n1p, ip=pe.ip, dp=pe.dp,
                        s_inter=pe.s_inter, s_n1p=pe.s_n1p, s_ip=pe.s_ip, w1_scale=s1, w2_scale=s2)
    if pe.ws1 is not None:
        out.ws1, out.ws1_scale = _quant_rows(pe.ws1)
        out.ws2, out.ws2_scale = _quant_rows(pe.ws2)
    return out


def dequantize_fp8(pe: PackedExperts) -> PackedExperts:
    """The weights an fp8 block computes with (q * scale), as a float32 PackedExperts."""
    f = PackedExperts(act=pe.act, d=pe.d, inter=pe.inter, E=pe.E,
                      w1=pe.w1.float() * pe.w1_scale[..., None], w2=pe.w2.float() * pe.w2_scale[..., None],
                      n1p=pe.n1p, ip=pe.ip, dp=pe.dp, s_inter=pe.s_inter, s_n1p=pe.s_n1p, s_ip=pe.s_ip)
    if pe.ws1 is not None:
        f.ws1 = pe.ws1.float() * pe.ws1_scale[..., None]
        f.ws2 = pe.ws2.float() * pe.ws2_scale[..., None]
    return f


def unpack_swiglu(pe: PackedExperts):
    """Inverse of pack_swiglu on float weights: (gate [E,I,d], up [E,I,d], down [E,d,I], shared)."""
    E, I, d, ip = pe.E, pe.inter, pe.d, pe.ip
    w = pe.w1.float().view(E, ip // 128, 2, 128, d)
    gate = w[:, :, 0].reshape(E, ip, d)[:, :I]
    up = w[:, :, 1].reshape(E, ip, d)[:, :I]
    down = pe.w2.float()[:, :d, :I]
    shared = None
    if pe.ws1 is not None:
        sip, Is = pe.s_ip, pe.s_inter
        s = pe.ws1.float().view(sip // 128, 2, 128, d)
        shared = (s[:, 0].reshape(sip, d)[:Is], s[:, 1].reshape(sip, d)[:Is], pe.ws2.float()[:d, :Is])
    return gate, up, down, shared


def _pack_glu_w1(gate: torch.Tensor, up: torch.Tensor) -> tuple[torch.Tensor, int]:
    """[E, I, d] gate / up -> [E, 2*Ip, d]: 256-row blocks of 128 gate rows, then the 128 up rows
    of the same intermediate channels (Ip = I rounded up to 128)."""
    E, I, d = gate.shape
    ip = _ceil(I, 128) * 128
    w = torch.zeros(E, ip // 128, 2, 128, d, dtype=gate.dtype, device=gate.device)
    g = torch.zeros(E, ip, d, dtype=gate.dtype, device=gate.device)
    u = torch.zeros(E, ip, d, dtype=gate.dtype, device=gate.device)
    g[:, :I] = gate
    u[:, :I] = up
    w[:, :, 0] = g.view(E, ip // 128, 128, d)
    w[:, :, 1] = u.view(E, ip // 128, 128, d)
    return w.view(E, 2 * ip, d).contiguous(), ip


def _pack_w2(down: torch.Tensor, ip: int) -> tuple[torch.Tensor, int]:
    """[E, d, I] -> [E, dp, ip] zero padded (dp = ceil(d/256)*256)."""
    E, d, I = down.shape
    dp = _ceil(d, 256) * 256
    w = torch.zeros(E, dp, ip, dtype=down.dtype, device=down.device)
    w[:, :d, :I] = down
    return w.contiguous(), dp


def pack_swiglu(gate, up, down, shared=None, dtype=torch.bfloat16, device="cuda") -> PackedExperts:
    """Qwen2MoeMLP experts: gate/up [E, I, d], down [E, d, I]; shared = (gate, up, down) of the
    shared expert ([Is, d], [Is, d], [d, Is]) or None."""
    gate = torch.as_tensor(gate).to(device=device, dtype=dtype)
    up = torch.as_tensor(up).to(device=device, dtype=dtype)
    down = torch.as_tensor(down).to(device=device, dtype=dtype)
    E, I, d = gate.shape
    w1, ip = _pack_glu_w1(gate, up)
    w2, dp = _pack_w2(down, ip)
    pe = PackedExperts(act=L.ACT_SWIGLU, d=d, inter=I, E=E, w1=w1, w2=w2, n1p=2 * ip, ip=ip, dp=dp)
    if shared is not None:
        sg, su, sd = (torch.as_tensor(t).to(device=device, dtype=dtype) for t in shared)
        ws1, sip = _pack_glu_w1(sg[None], su[None])
        ws2, _ = _pack_w2(sd[None], sip)
        pe.ws1, pe.ws2 = ws1[0].contiguous(), ws2[0].contiguous()
        pe.s_inter, pe.s_n1p, pe.s_ip = sg.shape[0], 2 * sip, sip
    return pe


def pack_relu(wi, wo, dtype=torch.bfloat16, device="cuda") -> PackedExperts:
    """Switch DenseActDense experts: wi [E, F, d], wo [E, d, F]."""
    wi = torch.as_tensor(wi).to(device=device, dtype=dtype)
    wo = torch.as_tensor(wo).to(device=device, dtype=dtype)
    E, F, d = wi.shape
    fp = _ceil(F, 256) * 256
    w1 = torch.zeros(E, fp, d, dtype=dtype, device=device)
    w1[:, :F] = wi
    w2, dp = _pack_w2(wo, fp)
    return PackedExperts(act=L.ACT_RELU, d=d, inter=F, E=E, w1=w1.contiguous(), w2=w2, n1p=fp, ip=fp, dp=dp)


# ----------------------------------------------------------------------------- plan (host C++)
def plan_harmony(meta: np.ndarray, expert_to_gpu, eq_tokens: int) -> np.ndarray:
    """S[G, E, G] from all-gathered counts meta[G, E] (dsca_plan_harmony)."""
    meta = np.ascontiguousarray(meta, dtype=np.int32)
    G, E = meta.shape
    e2g = np.ascontiguousarray(expert_to_gpu, dtype=np.int32)
    S = np.zeros((G, E, G), np.int32)
    L.call("dsca_plan_harmony", meta.ctypes.data, G, E, e2g.ctypes.data, int(eq_tokens), S.ctypes.data)
    return S


@dataclass
class Layout:
    num_groups: int
    group_expert: np.ndarray   # [ng]
    group_offsets: np.ndarray  # [ng + 1]
    recv_off: np.ndarray       # [G, E]
    send_base: np.ndarray      # [E, G]
    cum_split: np.ndarray      # [E, G]
    send_splits: np.ndarray    # [G]
    recv_splits: np.ndarray    # [G]


def plan_layout(S: np.ndarray, rank: int) -> Layout:
    S = np.ascontiguousarray(S, dtype=np.int32)
    G, E, _ = S.shape
    ng = ctypes.c_int(0)
    ge = np.zeros(E, np.int32)
    go = np.zeros(E + 1, np.int32)
    ro = np.zeros((G, E), np.int32)
    sb = np.zeros((E, G), np.int32)
    cs = np.zeros((E, G), np.int32)
    ss = np.zeros(G, np.int32)
    rs = np.zeros(G, np.int32)
    L.call("dsca_plan_layout", S.ctypes.data, G, E, rank, ctypes.byref(ng), ge.ctypes.data, go.ctypes.data,
           ro.ctypes.data, sb.ctypes.data, cs.ctypes.data, ss.ctypes.data, rs.ctypes.data)
    n = ng.value
    return Layout(n, ge[:n].copy(), go[:n + 1].copy(), ro, sb, cs, ss, rs)


def exchange_chunks(S: np.ndarray, lay: Layout, rank: int, send_buf, recv_buf, group=None, reverse=False):
    """Move the plan's (src, e, dst) chunks.  Forward: send_buf (sender layout) -> recv_buf
    (expert-major receive layout).  reverse=True moves expert outputs back: recv_buf (receive
    layout) -> send_buf (sender layout).  Chunks between one pair of ranks are posted in expert
    order on both sides, so NCCL pairs them in order.  Self chunks are device copies."""
    import torch.distributed as dist

    G, E, _ = S.shape
    ops = []
    for peer in range(G):
        for e in range(E):
            n_out = int(S[rank, e, peer])   # my tokens of e processed on peer
            n_in = int(S[peer, e, rank])    # peer's tokens of e processed here
            if peer == rank:
                if n_out:
                    a = int(lay.send_base[e, rank])
                    b = int(lay.recv_off[rank, e])
                    if not reverse:
                        recv_buf[b:b + n_out].copy_(send_buf[a:a + n_out])
                    else:
                        send_buf[a:a + n_out].copy_(recv_buf[b:b + n_out])
                continue
            if n_out:
                a = int(lay.send_base[e, peer])
                t = send_buf[a:a + n_out]
                ops.append(dist.P2POp(dist.irecv if reverse else dist.isend, t, peer, group))
            if n_in:
                b = int(lay.recv_off[peer, e])
                t = recv_buf[b:b + n_in]
                ops.append(dist.P2POp(dist.isend if reverse else dist.irecv, t, peer, group))
    if ops:
        for r in dist.batch_isend_irecv(ops):
            r.wait()


# ----------------------------------------------------------------------------- engine
class MoEEngine:
    """Runs one MoE block through libdsca_b200.

    router_weight [E, d] (router dtype == activation dtype, as the reference's nn.Linear
    requires); experts: PackedExperts; route_mode L.ROUTE_SWITCH_TOP1 or L.ROUTE_SOFTMAX_TOPK;
    shared_gate_weight [d] or None.  Multi-GPU: pass world > 1, a torch.distributed group and
    expert_to_gpu [E] (the placement), eq_tokens as in the reference scheduler.

    exchange = "p2p" (default): the fused NVLink path — counts, plan, dispatch and return all on
    the device over CUDA-IPC peer memory, no host synchronisation.  exchange = "nccl": the
    NCCL baseline (host plan, grouped send/recv).  p2p capacity is fixed by the first forward
    (max tokens over the ranks) or by reserve(tokens); wait_limit_ns bounds every device wait.
    """

    def __init__(self, router_weight: torch.Tensor, experts: PackedExperts, top_k: int, route_mode: int,
                 norm_topk: bool = False, shared_gate_weight: torch.Tensor | None = None,
                 rank: int = 0, world: int = 1, group=None, expert_to_gpu=None, eq_tokens: int = 150,
                 num_ctas: int = 0, exchange: str = "p2p", wait_limit_ns: int = 2_000_000_000,
                 cache_slots: int | None = None, device=None, initial_cache=None):
        lib = L.load()
        n_sms, is_sm100 = ctypes.c_int(0), ctypes.c_int(0)
        L.check(lib.dsca_device_info(ctypes.byref(n_sms), ctypes.byref(is_sm100)), "dsca_device_info")
        if experts.dtype == torch.bfloat16 and not is_sm100.value:
            raise RuntimeError("the bf16 expert path needs an sm_100 (B200) GPU")
        self.num_sms = n_sms.value
        n_experts = experts.E
        self.dtype = experts.dtype  # activation dtype (bf16 for fp8 weights)
        self.op_dtype = torch.float16 if experts.fp8 else self.dtype  # FFN operand dtype
        if experts.fp8 and world > 1 and exchange != "p2p":
            raise NotImplementedError("fp8 expert weights with more than one GPU need the fused exchange")
        self.device = torch.device(device) if device is not None else experts.w1.device
        # expert cache (the reference's expert_cache_size < num_experts): the routed weights stay
        # in pinned host memory and `cache_slots` device slots hold the ones being computed
        self.cache = None
        if cache_slots is not None:
            if experts.fp8 or (world > 1 and exchange != "p2p"):
                raise NotImplementedError("the expert cache takes bf16 / f32 weights and, with more than one "
                                          "GPU, the fused exchange")
            self.cache = ExpertCache.create(experts.w1, experts.w2, int(cache_slots), self.device, initial_cache)
            experts = replace(experts, w1=self.cache.w1, w2=self.cache.w2, E=int(cache_slots),
                              ws1=None if experts.ws1 is None else experts.ws1.to(self.device),
                              ws2=None if experts.ws2 is None else experts.ws2.to(self.device))
        # fp8 weights: True = the e4m3 weights go to the tensor cores unconverted (kind::f8f6f4)
        # against the tokens held as two e4m3 terms (dsca_split_rows); False = the weights are
        # converted to f16 inside the GEMM (tile_rows picks shared or tensor memory)
        self.fp8_split = bool(experts.fp8)
        # QoS planner constants (src/qosmoe/config.py:30-43), used by the expert-cache path
        self.qos_params = dict(alpha=1.0, beta=0.1, delta=0.5, target_batch=64.0, epsilon=1e-6, attention_mode=0)
        self.last_exec_plan = None
        self.last_loads = 0
        self.last_priority = None  # host copy of the expert priorities of the last cache-path forward
        self.experts = experts
        self.router_weight = router_weight.to(device=self.device, dtype=self.dtype).contiguous()
        self.E, self.d = self.router_weight.shape
        if self.E != n_experts or self.d != experts.d:
            raise ValueError("router and experts disagree on E / d")
        self.route_mode = route_mode
        self.top_k = 1 if route_mode == L.ROUTE_SWITCH_TOP1 else int(top_k)
        self.norm_topk = bool(norm_topk)
        self.shared_gate_weight = (None if shared_gate_weight is None else
                                   shared_gate_weight.reshape(-1).to(device=self.device, dtype=self.dtype).contiguous())
        if (self.shared_gate_weight is None) != (experts.ws1 is None):
            raise ValueError("shared expert and shared gate must be given together")
        # True (bf16 only): router logits on the tensor cores instead of the CUDA cores — exact
        # fixed-point accumulation on int8 tcgen05 MMAs (router_tc.cu).  On by default where the
        # one-kernel form applies (d <= 2048, at most 64 router rows), which measured faster than
        # the CUDA-core router (its fixed fp32 chunk order, the form for f32 and wider models)
        n_rows = self.E + (0 if self.shared_gate_weight is None else 1)
        self.router_tensor_cores = bool(self.dtype == torch.bfloat16 and self.d <= 2048 and n_rows <= 64)
        self._w_slices = self._w_exp = None
        self.rank, self.world, self.group = rank, world, group
        if expert_to_gpu is None:
            expert_to_gpu = default_expert_to_gpu(self.E, world)
        self.expert_to_gpu = np.asarray(expert_to_gpu, dtype=np.int32)
        self.eq_tokens = int(eq_tokens)
        self.num_ctas = num_ctas
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.exchange = exchange
        self.wait_limit_ns = int(wait_limit_ns)
        self._ep = None
        # one GPU through the fused exchange path (the rank is its own only peer): exercises the
        # plan / dispatch / return kernels without a second GPU
        self.ep_loopback = False
        # "overlap": routed GEMM2 stores locally and a return kernel sends the rows on a side
        # stream beside the shared-expert GEMM2; "fused": GEMM2's epilogue stores them remotely
        self.ep_return = "overlap"
        # SMs kept free of the shared-expert GEMMs while the side-stream copy kernels run beside
        # them (0: the copy kernels' small CTAs fit next to the persistent GEMM CTAs)
        self.ep_side_sms = 0
        # True: the router's last CTA computes counts / offsets / block bases (one launch);
        # False: the separate dsca_dispatch_scan launch does
        self.fuse_scan = True
        # bf16 expert GEMM tile form (dsca_ffn_args.tile_rows): 0 = default per GEMM,
        # 128 = single-CTA tiles, 256 = CTA-pair swap-AB tiles, 512 = CTA pairs with whole
        # 256-token blocks of the SwiGLU GEMM1 non-swapped; fp8 weights: 256 = converted into
        # tensor memory, else into shared memory
        self.tile_rows = 0
        # dsca_ffn_args.tile_order: bit 0 = routed and shared tiles of one launch interleaved
        # (else one segment after the other), bits 1 / 2 = shared / routed tiles weight-block major
        self.tile_order = 0
        # L2 policies of the GEMM loads (dsca_ffn_args.cache_hints): 0 = default, 1 = routed
        # weights evict-first, shared weights and token rows evict-last
        self.cache_hints = 0
        # routed GEMM tiles: L2 prefetch of the operand boxes this many K blocks ahead of the
        # shared-memory loads (dsca_ffn_args.cache_hints bits 8-15; 0 = off)
        self.l2_ahead = 0
        # one GPU: GEMM1 launched as a programmatic dependent of the permute (shared-expert tiles
        # overlap it; the routed tiles wait for it on the device)
        self.pdl = True
        # expert parallel: the QoS planner's token scores and expert priorities are computed on
        # every rank, summed over the ranks and order the routed experts' tiles (the reference's
        # world > 1 path always runs them, src/qosmoe/moe_layer.py:306-316,379-380,422-427)
        self.qos_order = True
        # where the QoS scores run at world > 1: "side" = on the side stream ahead of the plan,
        # which carries the priorities (the default); "parallel" = on a stream of their own, with
        # the priority exchange (dsca_ep_priority), beside the counts-only plan and the dispatch on
        # the side stream (the routed GEMM1 waits for both); "main" = on the main stream before
        # the shared GEMM1
        self.qos_stream = "side"
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._done_counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        # the QoS scores: first-choice counts accumulated by the router (zeroed again by the QoS
        # kernel) and the QoS kernel's own done counter
        self._first_counts = torch.zeros(self.E, dtype=torch.int32, device=self.device)
        # grouped GEMM tiles handed out by atomic tickets (dsca_ffn_args.tile_counters, 8 words;
        # every call leaves them zeroed) instead of the static schedule
        self.dynamic_tiles = True
        self._tile_ctr = torch.zeros(8, dtype=torch.int32, device=self.device)
        # GEMM2's shared-expert tiles start when GEMM1's are stored (dsca_ffn_args.shared_handoff;
        # one GPU, dynamic tiles)
        self.shared_handoff = True
        self._qos_done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ws = {}
        self.last_plan = None
        self.last_layout = None
        # when a list, forward() appends (name, cuda.Event) markers between its kernel launches
        # (and (name, start, end) of side-stream kernels to side_markers)
        self.markers = None
        self.side_markers = []

    def _mark(self, name: str):
        if self.markers is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.markers.append((name, ev))

    def _side_mark(self, name: str | None = None, start=None):
        """Timing of a side-stream kernel: call once before (returns the start event) and once
        after with its name; pairs land in side_markers when profiling is on."""
        if self.markers is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        if name is not None and start is not None:
            self.side_markers.append((name, start, ev))
        return ev

    @property
    def _qos_in_forward(self) -> bool:
        """Whether forward() runs the QoS scores (so the router accumulates their first-choice
        counts): the one-GPU expert-cache path, and the fused exchange with the QoS order."""
        if self.world == 1 and not self.ep_loopback:
            return self.cache is not None
        return self.exchange == "p2p" and self.qos_order

    @property
    def _uses_qos(self) -> bool:
        return self.cache is not None or ((self.world > 1 or self.ep_loopback) and self.exchange == "p2p")

    # -------------------------------------------------------------- workspace
    @property
    def _split(self) -> bool:
        return bool(self.experts.fp8 and self.fp8_split)

    def _workspace(self, T: int) -> dict:
        ws = self._ws.get((T, self._split))
        if ws is not None:
            return ws
        dev, dt, k, E, d = self.device, self.dtype, self.top_k, self.E, self.d
        nb = _ceil(T, L.ROUTER_TOKENS)
        pe = self.experts
        cap = max(T * k, 1)
        ws = dict(
            topk_w=torch.empty(T, k, dtype=torch.float32, device=dev),
            shared_gate=torch.empty(T, dtype=torch.float32, device=dev) if pe.ws1 is not None else None,
            block_hist=torch.empty(max(nb, 1), E, dtype=torch.int32, device=dev),
            local_rank=torch.empty(T, k, dtype=torch.int32, device=dev),
            counts=torch.empty(E, dtype=torch.int32, device=dev),
            offsets=torch.empty(E + 1, dtype=torch.int32, device=dev),
            block_base=torch.empty(max(nb, 1), E, dtype=torch.int32, device=dev),
            token_row=torch.empty(T, k, dtype=torch.int32, device=dev),
            token_score=torch.empty(T, dtype=torch.float32, device=dev) if self._uses_qos else None,
            qos_partial=(torch.empty(max(_ceil(T, 32), 1), E, dtype=torch.float32, device=dev)
                         if self._uses_qos else None),
            expert_priority=torch.empty(E, dtype=torch.float32, device=dev) if self._uses_qos else None,
            # fp8 weights: the FFN operands (rows, shared input, intermediates) are f16
            hs=torch.empty(T, pe.s_ip, dtype=self.op_dtype, device=dev) if pe.ws1 is not None else None,
            ys=torch.empty(T, d, dtype=dt, device=dev) if pe.ws1 is not None else None,
            x_f16=torch.empty(T, d, dtype=torch.float16, device=dev) if (pe.fp8 and pe.ws1 is not None) else None,
        )
        if self._split:
            # two-term e4m3 token rows ([hi | lo], kd bytes each) with 1 / s per row; bf16
            # intermediates, split again for GEMM2
            kd = _ceil(d, 128) * 128
            ws["x_f16"] = None
            if pe.ws1 is not None:
                ws.update(hs=torch.empty(T, pe.s_ip, dtype=torch.bfloat16, device=dev),
                          x_q=torch.empty(T, 2 * kd, dtype=torch.uint8, device=dev),
                          x_scale=torch.empty(T, dtype=torch.float32, device=dev),
                          hsq=torch.empty(T, 2 * pe.s_ip, dtype=torch.uint8, device=dev),
                          hs_scale=torch.empty(T, dtype=torch.float32, device=dev))
            if self.world == 1:
                ws.update(a=torch.empty(cap, 2 * kd, dtype=torch.uint8, device=dev),
                          a_scale=torch.empty(cap, dtype=torch.float32, device=dev),
                          h=torch.empty(cap, pe.ip, dtype=torch.bfloat16, device=dev),
                          hq=torch.empty(cap, 2 * pe.ip, dtype=torch.uint8, device=dev),
                          h_scale=torch.empty(cap, dtype=torch.float32, device=dev),
                          y=torch.empty(cap, d, dtype=dt, device=dev))
        elif self.world == 1:
            ws.update(a=torch.empty(cap, d, dtype=self.op_dtype, device=dev),
                      h=torch.empty(cap, pe.ip, dtype=self.op_dtype, device=dev),
                      y=torch.empty(cap, d, dtype=dt, device=dev))
        self._ws = {(T, self._split): ws}  # keep one shape resident
        return ws

    # -------------------------------------------------------------- kernel steps
    def _router_tc_buffers(self, T: int) -> dict:
        """Tensor-core router: the sliced router rows (once), and for d > 2048 the per-call scratch for
        T tokens."""
        if self.dtype != torch.bfloat16:
            raise ValueError("the tensor-core router takes bf16 inputs")
        d16 = _ceil(self.d, 16) * 16
        if self._w_slices is None:
            rows = self.router_weight if self.shared_gate_weight is None else torch.cat(
                [self.router_weight, self.shared_gate_weight[None]], 0)
            self._w_rows = rows.contiguous()
            self._w_slices = torch.empty(3, 64, d16, dtype=torch.int8, device=self.device)
            self._w_exp = torch.empty(64, dtype=torch.int32, device=self.device)
            L.call("dsca_router_pack_i8", _ptr(self._w_rows), self._w_rows.shape[0], self.d, _ptr(self._w_slices),
                   _ptr(self._w_exp), _stream())
        if self.d <= 2048:  # the fused kernel: no scratch
            return {}
        tc = getattr(self, "_tc_ws", None)
        if tc is None or tc["x_exp"].shape[0] != T:
            dev = self.device
            tc = dict(x_slices=torch.empty(3, T, d16, dtype=torch.int8, device=dev),
                      x_exp=torch.empty(T, dtype=torch.int32, device=dev),
                      logits_f32=torch.empty(T, 64, dtype=torch.float32, device=dev))
            self._tc_ws = tc
        return tc

    def _route(self, x: torch.Tensor, ws: dict):
        T = x.shape[0]
        a = L.RouterArgs()
        a.x, a.w_router = _ptr(x), _ptr(self.router_weight)
        a.w_shared_gate = _ptr(self.shared_gate_weight)
        a.T, a.d, a.E, a.top_k = T, self.d, self.E, self.top_k
        a.dtype = _dt(self.dtype)
        a.mode = self.route_mode
        a.norm_topk = int(self.norm_topk)
        a.weight_round_bf16 = int(self.dtype == torch.bfloat16)
        a.logits, a.topk_ids, a.topk_w = _ptr(ws["logits"]), _ptr(ws["topk_ids"]), _ptr(ws["topk_w"])
        a.expert_index = _ptr(ws["expert_index"])
        a.shared_gate = _ptr(ws["shared_gate"])
        a.block_hist, a.local_rank = _ptr(ws["block_hist"]), _ptr(ws["local_rank"])
        if self._qos_in_forward:
            a.first_counts = _ptr(self._first_counts)
        if self.fuse_scan:
            a.counts, a.offsets, a.block_base = _ptr(ws["counts"]), _ptr(ws["offsets"]), _ptr(ws["block_base"])
            a.done_counter = _ptr(self._done_counter)
        if self.router_tensor_cores:
            tc = self._router_tc_buffers(T)
            a.w_slices, a.w_exp = _ptr(self._w_slices), _ptr(self._w_exp)
            if tc:
                a.x_slices, a.x_exp, a.logits_f32 = _ptr(tc["x_slices"]), _ptr(tc["x_exp"]), _ptr(tc["logits_f32"])
            a.err = _ptr(self.err)
        L.call("dsca_router_topk", ctypes.byref(a), _stream())
        self._mark("router")
        if self.fuse_scan:
            return
        s = L.ScanArgs()
        s.block_hist, s.nblocks, s.E = _ptr(ws["block_hist"]), _ceil(T, L.ROUTER_TOKENS), self.E
        s.counts, s.offsets, s.block_base = _ptr(ws["counts"]), _ptr(ws["offsets"]), _ptr(ws["block_base"])
        L.call("dsca_dispatch_scan", ctypes.byref(s), _stream())

    def _permute(self, x, ws, out, capacity, G=1, cum_split=None, dest_base=None):
        p = L.PermuteArgs()
        p.x, p.T, p.d, p.E, p.top_k, p.dtype = _ptr(x), x.shape[0], self.d, self.E, self.top_k, _dt(self.dtype)
        p.topk_ids, p.local_rank, p.block_base = _ptr(ws["topk_ids"]), _ptr(ws["local_rank"]), _ptr(ws["block_base"])
        p.offsets = _ptr(ws["offsets"])
        p.G, p.cum_split, p.dest_base = G, _ptr(cum_split), _ptr(dest_base)
        p.capacity, p.out, p.token_row, p.err = capacity, _ptr(out), _ptr(ws["token_row"]), _ptr(self.err)
        if self._split:
            p.out_e4m3, p.out_scale = 1, _ptr(ws["a_scale"])
            p.x_q, p.x_scale = _ptr(ws.get("x_q")), _ptr(ws.get("x_scale"))
        else:
            p.out_f16 = int(self.experts.fp8)
            p.x_f16 = _ptr(ws.get("x_f16"))
        L.call("dsca_permute", ctypes.byref(p), _stream())

    def _split_rows(self, src, rows, K, dst, inv_scale, rows_dev=0):
        """dsca_split_rows: bf16 rows [rows, K] -> two-term e4m3 rows and 1 / s."""
        a = L.SplitArgs()
        a.src, a.ld, a.rows, a.K = _ptr(src), src.shape[1], rows, K
        a.rows_dev, a.dst, a.inv_scale = rows_dev, _ptr(dst), _ptr(inv_scale)
        L.call("dsca_split_rows", ctypes.byref(a), _stream())

    def _ffn(self, x, ws, a, h, y, capacity, num_groups, group_offsets, group_weight, ep_ctx=None,
             after_permute=False):
        if self.markers is not None:
            # time GEMM1 and GEMM2 as separate launches
            self._ffn_call(x, ws, a, h, y, capacity, num_groups, group_offsets, group_weight, 1, ep_ctx,
                           after_permute=after_permute)
            self._mark("gemm1")
            self._ffn_call(x, ws, a, h, y, capacity, num_groups, group_offsets, group_weight, 2, ep_ctx)
            self._mark("gemm2")
        else:
            self._ffn_call(x, ws, a, h, y, capacity, num_groups, group_offsets, group_weight, 3, ep_ctx,
                           after_permute=after_permute)

    def _ffn_call(self, x, ws, a, h, y, capacity, num_groups, group_offsets, group_weight, phases, ep_ctx=None,
                  segments=3, num_ctas=None, after_permute=False, group_order=None, split=None):
        """`split` (two-term fp8 path): the routed rows' (a_scale, hq, h_scale); default the one-GPU
        workspace's."""
        pe = self.experts  # with an expert cache: w1 / w2 are the device slots
        f = L.FfnArgs()
        f.dtype, f.act, f.d = (L.F8E4M3 if pe.fp8 else _dt(self.dtype)), pe.act, self.d
        f.n1p, f.ip, f.dp = pe.n1p, pe.ip, pe.dp
        f.num_groups, f.group_offsets, f.group_weight = num_groups, _ptr(group_offsets), _ptr(group_weight)
        f.num_experts_w, f.capacity = pe.E, capacity
        f.a, f.w1, f.w2, f.h, f.y = _ptr(a), _ptr(pe.w1), _ptr(pe.w2), _ptr(h), _ptr(y)
        if pe.ws1 is not None:
            xs = (ws["x_q"] if self._split else ws["x_f16"]) if pe.fp8 else x
            f.shared_rows, f.shared_n1p, f.shared_ip = x.shape[0], pe.s_n1p, pe.s_ip
            f.xs, f.ws1, f.ws2, f.hs, f.ys = _ptr(xs), _ptr(pe.ws1), _ptr(pe.ws2), _ptr(ws["hs"]), _ptr(ws["ys"])
        if pe.fp8:
            f.w1_scale, f.w2_scale = _ptr(pe.w1_scale), _ptr(pe.w2_scale)
            f.ws1_scale, f.ws2_scale = _ptr(pe.ws1_scale), _ptr(pe.ws2_scale)
        if self._split:
            a_scale, hq, h_scale = split if split is not None else (ws["a_scale"], ws["hq"], ws["h_scale"])
            f.f8_split, f.a_scale, f.hq, f.h_scale = 1, _ptr(a_scale), _ptr(hq), _ptr(h_scale)
            if pe.ws1 is not None:
                f.xs_scale, f.hsq, f.hs_scale = _ptr(ws["x_scale"]), _ptr(ws["hsq"]), _ptr(ws["hs_scale"])
        f.err, f.num_ctas, f.phases = _ptr(self.err), self.num_ctas if num_ctas is None else num_ctas, phases
        f.tile_rows = self.tile_rows
        f.tile_order = self.tile_order
        f.cache_hints = self.cache_hints | (self.l2_ahead << 8)
        f.group_order = _ptr(group_order)
        f.ep_ctx = _ptr(ep_ctx)
        f.segments = segments
        # GEMM1 directly after the permute: its shared-expert tiles overlap the permute
        f.pdl_after_permute = int(after_permute and self.pdl)
        f.tile_counters = _ptr(self._tile_ctr) if self.dynamic_tiles else None
        f.shared_handoff = int(self.shared_handoff and self.dynamic_tiles)
        L.call("dsca_grouped_ffn", ctypes.byref(f), _stream())

    def _combine(self, ws, y, rows, after_ffn=False):
        c = L.CombineArgs()
        # directly after dsca_grouped_ffn on this stream: a programmatic dependent of GEMM2
        c.pdl = int(after_ffn and self.pdl)
        c.T, c.d, c.top_k, c.dtype = ws["out"].shape[0], self.d, self.top_k, _dt(self.dtype)
        c.y, c.token_row, c.topk_w = _ptr(y), _ptr(ws["token_row"]), _ptr(ws["topk_w"])
        c.ys, c.shared_gate = _ptr(ws["ys"]), _ptr(ws["shared_gate"])
        c.rows, c.out, c.err = rows, _ptr(ws["out"]), _ptr(self.err)
        L.call("dsca_combine", ctypes.byref(c), _stream())

    # -------------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, qos: QoSInputs | None = None) -> dict:
        """x [T, d] (activation dtype, on this engine's device).  Returns a dict with the fresh
        results out [T, d], logits [T, E], topk_ids [T, k] and expert_index [T] (int64), plus
        views of the reused scratch (topk_w, counts, token_row, ...) valid until the next call.
        `qos`: the planner's per-token inputs, read only with an expert cache (they order the
        experts and choose the slots, never the result)."""
        if x.dim() != 2 or x.shape[1] != self.d:
            raise ValueError(f"expected [T, {self.d}] input, got {tuple(x.shape)}")
        x = x.to(dtype=self.dtype).contiguous()
        T = x.shape[0]
        ws = dict(self._workspace(T))
        dev, k = self.device, self.top_k
        # results are fresh tensors (the caller keeps them); scratch above is reused
        ws.update(out=torch.empty(T, self.d, dtype=self.dtype, device=dev),
                  logits=torch.empty(T, self.E, dtype=self.dtype, device=dev),
                  topk_ids=torch.empty(T, k, dtype=torch.int32, device=dev),
                  expert_index=torch.empty(T, dtype=torch.int64, device=dev))
        if T == 0:
            return ws
        self._mark("start")
        self._route(x, ws)
        self._mark("scan")
        if self.world == 1 and self.cache is not None:
            return self._forward_cached(x, ws, qos)
        if self.world == 1 and not self.ep_loopback:
            cap = ws["a"].shape[0]
            self._permute(x, ws, ws["a"], cap)
            self._mark("permute")
            self._ffn(x, ws, ws["a"], ws["h"], ws["y"], cap, self.E, ws["offsets"], None, after_permute=True)
            self._combine(ws, ws["y"], cap, after_ffn=self.markers is None)
            self._mark("combine")
            return ws
        return self._forward_ep(x, ws, qos)

    # -------------------------------------------------------------- expert cache path
    def _qos(self, x, ws, qos: QoSInputs | None):
        """dsca_qos_priority: token scores and expert priorities into the workspace."""
        T = x.shape[0]
        q = qos or QoSInputs()
        dev = self.device

        def vec(v):
            v = match_token_length(v, T)
            return None if v is None else v.to(device=dev, dtype=torch.float32).contiguous()

        xp = q.x_prev
        if xp is not None:
            xp = xp.reshape(-1, xp.shape[-1]) if xp.dim() > 1 else xp
            xp = xp.to(device=dev, dtype=self.dtype).contiguous() if tuple(xp.shape) == tuple(x.shape) else None
        seq, rem, val = vec(q.seq_priority), vec(q.remaining), vec(q.valid)
        a = L.QosArgs()
        a.x, a.x_prev, a.logits, a.dtype = _ptr(x), _ptr(xp), _ptr(ws["logits"]), _dt(self.dtype)
        a.topk_ids, a.seq_priority, a.remaining, a.valid = _ptr(ws["topk_ids"]), _ptr(seq), _ptr(rem), _ptr(val)
        a.T, a.d, a.E, a.top_k = T, self.d, self.E, self.top_k
        p = self.qos_params
        a.attention_mode = int(p["attention_mode"])
        a.alpha, a.beta, a.delta = p["alpha"], p["beta"], p["delta"]
        a.target_batch, a.epsilon = p["target_batch"], p["epsilon"]
        a.token_score, a.expert_priority, a.err = _ptr(ws["token_score"]), _ptr(ws["expert_priority"]), _ptr(self.err)
        # one kernel; n(e) from the router of this forward (see _route)
        a.first_counts = _ptr(self._first_counts) if self._qos_in_forward else None
        a.partial, a.done_counter = _ptr(ws["qos_partial"]), _ptr(self._qos_done)
        L.call("dsca_qos_priority", ctypes.byref(a), _stream())
        # keep the per-token vectors alive until the kernel has read them
        ws["_qos_keep"] = (xp, seq, rem, val)

    def _forward_cached(self, x, ws, qos):
        """One GPU, routed experts in `cache.slots` device slots: the shared expert first, then
        the QoS plan's experts one grouped-GEMM launch each, every expert copied into its planned
        slot (load stream) before its GEMM and a slot reused only after its last reader."""
        cache = self.cache
        cap = ws["a"].shape[0]
        self._permute(x, ws, ws["a"], cap)
        self._mark("permute")
        if self.experts.ws1 is not None:
            self._ffn_call(x, ws, ws["a"], ws["h"], ws["y"], cap, 1, ws["offsets"], None, 3, segments=2)
        self._qos(x, ws, qos)
        # the plan decides what crosses PCIe: the host reads counts and priorities (as the
        # reference does with .item() per expert)
        counts = ws["counts"].cpu().numpy()
        prio = ws["expert_priority"].cpu().numpy()
        self.last_priority = prio
        plan = build_exec_plan(np.nonzero(counts > 0)[0], prio, cache.resident, cache.slots)
        loads0 = cache.loads
        cur = torch.cuda.current_stream(self.device)
        need = set(plan.need_loading)
        for e, s in zip(plan.expert_order, plan.slot_idxs):
            if e in need:
                cache.load(e, s)
            cur.wait_event(cache.loaded[s])
            self._ffn_call(x, ws, ws["a"], ws["h"], ws["y"], cap, 1, ws["offsets"][e:e + 2],
                           cache.slot_ids[s:s + 1], 3, segments=1)
            cache.free[s].record(cur)
        self.last_exec_plan = plan
        self.last_loads = cache.loads - loads0
        self._mark("experts")
        self._combine(ws, ws["y"], cap)
        self._mark("combine")
        return ws

    def _forward_ep(self, x, ws, qos=None):
        if self.exchange == "p2p":
            return self._forward_p2p(x, ws, qos)
        return self._forward_nccl(x, ws)

    def last_priority_host(self):
        """Expert priorities of the last forward on the host (the summed priorities with more than
        one GPU), or None when that forward computed none.  Synchronises."""
        if self.cache is not None and self.world == 1 and not self.ep_loopback:
            return self.last_priority
        if self._ep is not None and self.qos_order:
            return self.read_qos_order()[1]
        return None

    # -------------------------------------------------------------- fused NVLink path
    def reserve(self, tokens: int):
        """Collective (every rank calls it): size the symmetric region for `tokens` tokens per
        rank (max over the ranks is used) and map every peer's region."""
        self._p2p_setup(tokens)

    def _p2p_setup(self, T: int):
        import torch.distributed as dist

        lib = L.load()
        G, me, k, d, dev = self.world, self.rank, self.top_k, self.d, self.device
        if G > L.MAX_GPUS or self.E > L.MAX_EXPERTS:
            raise ValueError("the p2p exchange supports up to 8 GPUs and 64 experts")
        if G > 1:
            t = torch.tensor([T], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            T = int(t.item())
        T_cap = max(T, 1)
        esz = 2 if self.dtype == torch.bfloat16 else 4
        recv_cap, ret_cap = G * T_cap * k, T_cap * k
        off_flags, off_meta = 0, 256
        off_recv = 256 + 2 * 4 * L.MAX_GPUS * L.MAX_EXPERTS  # counts, then priorities
        off_recv = _ceil(off_recv, 256) * 256
        off_ret = _ceil(off_recv + recv_cap * d * esz, 256) * 256
        total = off_ret + ret_cap * d * esz
        region = ctypes.c_void_p()
        L.call("dsca_ep_region_alloc", ctypes.c_size_t(total), ctypes.byref(region))
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_size_t(0)
        L.call("dsca_ipc_export", region, handle, ctypes.byref(off))
        allh = [(bytes(handle), int(off.value))]
        if G > 1:
            allh = [None] * G
            dist.all_gather_object(allh, (bytes(handle), int(off.value)), group=self.group)
        bases, imported = [], []
        for p in range(G):
            if p == me:
                bases.append(region.value)
                continue
            h = (ctypes.c_char * 64).from_buffer_copy(allh[p][0])
            ptr = ctypes.c_void_p()
            L.call("dsca_ipc_import", h, ctypes.c_size_t(allh[p][1]), ctypes.byref(ptr))
            bases.append(ptr.value)
            imported.append((ptr.value, allh[p][1]))
        s = L.EpSetup()
        s.G, s.E, s.me, s.d, s.elem_bytes = G, self.E, me, d, esz
        s.recv_capacity, s.ret_capacity, s.eq_tokens, s.start_epoch = recv_cap, ret_cap, self.eq_tokens, 0
        e2g = np.ascontiguousarray(self.expert_to_gpu, dtype=np.int32)
        s.expert_to_gpu = e2g.ctypes.data
        for p in range(G):
            s.flags[p] = bases[p] + off_flags
            s.meta[p] = bases[p] + off_meta
            s.recv[p] = bases[p] + off_recv
            s.ret[p] = bases[p] + off_ret
        ctx = torch.empty(int(lib.dsca_ep_ctx_bytes()), dtype=torch.uint8, device=dev)
        L.call("dsca_ep_init", _ptr(ctx), ctypes.byref(s), _stream())
        torch.cuda.synchronize(dev)
        if G > 1:
            dist.barrier(group=self.group)  # every region is zeroed and mapped before anyone stores
        dt = self.dtype
        split = {}
        if self._split:
            # the received bf16 rows and the intermediates as two-term e4m3 rows (dsca_split_rows)
            kd, ip = _ceil(d, 128) * 128, self.experts.ip
            split = dict(aq=torch.empty(recv_cap, 2 * kd, dtype=torch.uint8, device=dev),
                         a_scale=torch.empty(recv_cap, dtype=torch.float32, device=dev),
                         hq=torch.empty(recv_cap, 2 * ip, dtype=torch.uint8, device=dev),
                         h_scale=torch.empty(recv_cap, dtype=torch.float32, device=dev))
        self._ep = dict(
            region=region.value, imported=imported, ctx=ctx, T_cap=T_cap, recv_cap=recv_cap, ret_cap=ret_cap,
            recv=_DevPtr.tensor(region.value + off_recv, (recv_cap, d), dt, dev),
            ret=_DevPtr.tensor(region.value + off_ret, (ret_cap, d), dt, dev),
            h=torch.empty(recv_cap, self.experts.ip, dtype=torch.bfloat16 if self._split else self.op_dtype,
                          device=dev),
            y=torch.empty(recv_cap, d, dtype=dt, device=dev),
            side=torch.cuda.Stream(device=dev),
            qos_side=torch.cuda.Stream(device=dev),
            group_offsets=int(lib.dsca_ep_group_offsets(_ptr(ctx)) or 0),
            group_order=int(lib.dsca_ep_group_order(_ptr(ctx)) or 0),
            bytes=total, split_fp8=self._split, **split)

    def _forward_p2p(self, x, ws, qos=None):
        """ep_return = "overlap": main stream shared GEMM1 -> [dispatch done] routed GEMM1 ->
        routed GEMM2 -> shared GEMM2 -> [return done] combine; side stream: plan and dispatch
        (beside the shared GEMM1) and the return kernel (beside the shared GEMM2).
        ep_return = "fused": main stream shared GEMM1 -> shared GEMM2 -> [dispatch done] routed
        GEMM1 -> routed GEMM2 whose epilogue stores every output row straight into the return
        buffer of the rank that sent it (the return all-to-all fused into the GEMM, tile by tile)
        -> [return done] combine; side stream: plan and dispatch beside both shared GEMMs."""
        T = x.shape[0]
        if self._ep is None:
            self._p2p_setup(T)
        ep = self._ep
        if T > ep["T_cap"]:
            raise RuntimeError(f"{T} tokens exceed the reserved {ep['T_cap']} per rank (call reserve())")
        lib, ctx, err = L.load(), _ptr(ep["ctx"]), _ptr(self.err)
        main, side = torch.cuda.current_stream(), ep["side"]
        # the plan (counts exchange + harmony) and the dispatch run on the side stream, beside the
        # shared-expert GEMM1, which needs neither
        prio = None
        parallel = self.qos_order and self.qos_stream == "parallel" and self.cache is None
        prio_done = None
        if self.qos_order and self.qos_stream == "main":
            # the QoS scores alone on the GPU, before the shared-expert GEMM1 fills it (beside it
            # they share its SMs and lengthen the side stream's chain to the dispatch)
            self._qos(x, ws, qos)
            prio = ws["expert_priority"]
            self._mark("qos")
        routed = torch.cuda.Event()
        routed.record(main)
        side.wait_event(routed)
        if parallel:
            # the QoS scores and the priority exchange on their own stream: the plan and the
            # dispatch need only the counts
            qs = ep["qos_side"]
            qs.wait_event(routed)
            with torch.cuda.stream(qs):
                t0 = self._side_mark()
                self._qos(x, ws, qos)
                self._side_mark("qos", t0)
                t0 = self._side_mark()
                L.check(lib.dsca_ep_priority(ctx, _ptr(ws["expert_priority"]), self.wait_limit_ns, err, _stream()),
                        "dsca_ep_priority")
                self._side_mark("priority", t0)
                prio_done = torch.cuda.Event()
                prio_done.record(qs)
        with torch.cuda.stream(side):
            if self.qos_order and not parallel and self.qos_stream != "main":
                t0 = self._side_mark()
                self._qos(x, ws, qos)
                prio = ws["expert_priority"]
                self._side_mark("qos", t0)
            t0 = self._side_mark()
            if parallel:
                L.check(lib.dsca_ep_plan_counts(ctx, _ptr(ws["counts"]), self.wait_limit_ns, err, _stream()),
                        "dsca_ep_plan_counts")
            else:
                L.check(lib.dsca_ep_plan(ctx, _ptr(ws["counts"]), _ptr(prio), self.wait_limit_ns, err, _stream()),
                        "dsca_ep_plan")
            self._side_mark("plan", t0)
            t0 = self._side_mark()
            a = L.EpDispatchArgs()
            a.x, a.T, a.d, a.top_k, a.dtype = _ptr(x), T, self.d, self.top_k, _dt(self.dtype)
            a.topk_ids, a.local_rank = _ptr(ws["topk_ids"]), _ptr(ws["local_rank"])
            a.block_base, a.ctx, a.token_row, a.err = _ptr(ws["block_base"]), ctx, _ptr(ws["token_row"]), err
            if not self._split:  # the two-term fp8 path sends bf16 rows and splits them on arrival
                a.out_f16, a.x_f16 = int(self.experts.fp8), _ptr(ws.get("x_f16"))
            L.call("dsca_ep_dispatch", ctypes.byref(a), _stream())
            self._side_mark("dispatch", t0)
            dispatched = torch.cuda.Event()
            dispatched.record(side)
        has_shared = self.experts.ws1 is not None
        kw = {}
        if self._split:
            kw = dict(split=(ep["a_scale"], ep["hq"], ep["h_scale"]))
            if has_shared:
                self._split_rows(x, T, self.d, ws["x_q"], ws["x_scale"])
        args = (x, ws, ep["aq"] if self._split else ep["recv"], ep["h"], ep["y"], ep["recv_cap"], self.E,
                ep["group_offsets"], None)
        # the fp8-weight GEMM has no remote-store epilogue: its routed rows go back by the return kernel
        fused = self.ep_return == "fused" and not self.experts.fp8
        side_ctas = max(2, self.num_sms - self.ep_side_sms) if self.ep_side_sms > 0 else None
        if has_shared:
            self._ffn_call(*args, 1, segments=2, num_ctas=side_ctas, **kw)
            self._mark("gemm1_shared")
            if fused:
                self._ffn_call(*args, 2, segments=2, num_ctas=side_ctas, **kw)
                self._mark("gemm2_shared")
        main.wait_event(dispatched)
        L.check(lib.dsca_ep_wait(ctx, 1, self.wait_limit_ns, err, _stream()), "dsca_ep_wait")
        self._mark("wait_dispatch")
        if self._split:
            # the received rows (as many as the plan's receive offsets hold) as two-term rows
            self._split_rows(ep["recv"], ep["recv_cap"], self.d, ep["aq"], ep["a_scale"],
                             rows_dev=ep["group_offsets"] + 4 * self.E)
            self._mark("split_received")
        if self.cache is not None:
            return self._forward_p2p_cached(x, ws, ep, args, has_shared, side_ctas)
        order = ep["group_order"] if self.qos_order else None
        if prio_done is not None:
            main.wait_event(prio_done)
        self._ffn_call(*args, 1, segments=1, group_order=order, **kw)
        self._mark("gemm1_routed")
        if fused:
            self._ffn_call(*args, 2, ep_ctx=ep["ctx"], segments=1, group_order=order)
            self._mark("gemm2_routed_fused")
        else:
            self._ffn_call(*args, 2, segments=1, group_order=order, **kw)
            self._mark("gemm2_routed")
            computed = torch.cuda.Event()
            computed.record(main)
            side.wait_event(computed)
            with torch.cuda.stream(side):
                t0 = self._side_mark()
                L.check(lib.dsca_ep_return(ctx, _ptr(ep["y"]), self.d, _dt(self.dtype), ep["recv_cap"], err,
                                           _stream()), "dsca_ep_return")
                self._side_mark("return", t0)
                returned = torch.cuda.Event()
                returned.record(side)
            if has_shared:
                self._ffn_call(*args, 2, segments=2, num_ctas=side_ctas, **kw)
                self._mark("gemm2_shared")
            main.wait_event(returned)
        L.check(lib.dsca_ep_wait(ctx, 2, self.wait_limit_ns, err, _stream()), "dsca_ep_wait")
        self._mark("wait_return")
        self._combine(ws, ep["ret"], ep["ret_cap"])
        self._mark("combine")
        return ws

    def _forward_p2p_cached(self, x, ws, ep, args, has_shared, side_ctas):
        """Expert parallel with an expert cache (the reference runs its cache path on every rank,
        src/qosmoe/async_cpu.py:98-256, execute_job :175): once the dispatched rows are here,
        the host reads which experts received rows and the summed priorities (one
        synchronisation, as the reference's .tolist() / .item() calls), plans the order and the
        slots with build_exec_plan, and runs each expert's GEMMs from its slot, loading the
        experts that are not cached on the load stream; then the return kernel, the return wait
        and the combine.  Every expert is computed from its own weights, so the output equals the
        resident path's."""
        lib, ctx, err = L.load(), _ptr(ep["ctx"]), _ptr(self.err)
        cache = self.cache
        if has_shared and not (self.ep_return == "fused" and not self.experts.fp8):
            self._ffn_call(*args, 2, segments=2, num_ctas=side_ctas)
            self._mark("gemm2_shared")
        torch.cuda.current_stream(self.device).synchronize()
        goff = _DevPtr.tensor(ep["group_offsets"], (self.E + 1,), torch.int32, self.device).cpu().numpy()
        if self.qos_order:
            prio = _DevPtr.tensor(ep["group_order"] + 4 * L.MAX_EXPERTS, (self.E,), torch.float32,
                                  self.device).cpu().numpy()
        else:
            prio = np.zeros(self.E, np.float32)
        self.last_priority = prio
        active = np.nonzero(np.diff(goff) > 0)[0]
        plan = build_exec_plan(active, prio, cache.resident, cache.slots)
        loads0 = cache.loads
        cur = torch.cuda.current_stream(self.device)
        need = set(plan.need_loading)
        rows = ep["recv_cap"]
        for e, s in zip(plan.expert_order, plan.slot_idxs):
            if e in need:
                cache.load(e, s)
            cur.wait_event(cache.loaded[s])
            self._ffn_call(x, ws, ep["recv"], ep["h"], ep["y"], rows, 1, ep["group_offsets"] + 4 * int(e),
                           cache.slot_ids[s:s + 1], 3, segments=1)
            cache.free[s].record(cur)
        self.last_exec_plan = plan
        self.last_loads = cache.loads - loads0
        self._mark("experts")
        L.check(lib.dsca_ep_return(ctx, _ptr(ep["y"]), self.d, _dt(self.dtype), ep["recv_cap"], err, _stream()),
                "dsca_ep_return")
        self._mark("return")
        L.check(lib.dsca_ep_wait(ctx, 2, self.wait_limit_ns, err, _stream()), "dsca_ep_wait")
        self._mark("wait_return")
        self._combine(ws, ep["ret"], ep["ret_cap"])
        self._mark("combine")
        return ws

    def read_qos_order(self):
        """(execution order [E], summed priorities [E]) of the last expert-parallel forward (host
        copies; synchronises)."""
        if self._ep is None:
            return None, None
        ctx = self._ep["ctx"]
        torch.cuda.synchronize(self.device)
        order = _DevPtr.tensor(self._ep["group_order"], (self.E,), torch.int32, self.device).cpu().numpy()
        prio = _DevPtr.tensor(self._ep["group_order"] + 4 * L.MAX_EXPERTS, (self.E,), torch.float32,
                              self.device).cpu().numpy()
        del ctx
        return order, prio

    def read_plan(self):
        """(S [G, E, G], rows received here) of the last forward (host copy; synchronises)."""
        if self.exchange == "nccl" or self._ep is None:
            S = self.last_plan
            return S, (int(self.last_layout.group_offsets[-1]) if self.last_layout is not None else 0)
        S = np.zeros((L.MAX_GPUS, L.MAX_EXPERTS, L.MAX_GPUS), np.int32)
        rt = np.zeros(1, np.int32)
        L.call("dsca_ep_read_plan", _ptr(self._ep["ctx"]), S.ctypes.data, rt.ctypes.data, _stream())
        return S[:self.world, :self.E, :self.world].copy(), int(rt[0])

    def close(self):
        """Unmap the peers' regions and free this rank's (collective: every rank calls it, after
        its last forward)."""
        if self._ep is None:
            return
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer stores into our region any more
        for ptr, off in self._ep["imported"]:
            L.load().dsca_ipc_close(ctypes.c_void_p(ptr), ctypes.c_size_t(off))
        if self.world > 1:
            dist.barrier(group=self.group)  # every peer has unmapped ours
        L.load().dsca_ep_region_free(ctypes.c_void_p(self._ep["region"]))
        self._ep = None

    # -------------------------------------------------------------- NCCL baseline path
    def _forward_nccl(self, x, ws):
        import torch.distributed as dist

        G, rank, E, d, dt, dev = self.world, self.rank, self.E, self.d, self.dtype, self.device
        meta = torch.empty(G, E, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(meta, ws["counts"], group=self.group)
        meta_h = meta.cpu().numpy()
        S = plan_harmony(meta_h, self.expert_to_gpu, self.eq_tokens)
        lay = plan_layout(S, rank)
        self.last_plan, self.last_layout = S, lay
        send_total = int(lay.send_splits.sum())
        recv_total = int(lay.recv_splits.sum())
        small = torch.from_numpy(np.concatenate([lay.cum_split.reshape(-1), lay.send_base.reshape(-1),
                                                 lay.group_offsets, lay.group_expert])).to(dev, non_blocking=True)
        n = E * G
        cum_split, send_base = small[:n], small[n:2 * n]
        ng = lay.num_groups
        group_offsets = small[2 * n:2 * n + ng + 1]
        group_expert = small[2 * n + ng + 1:]
        send_buf = torch.empty(max(send_total, 1), d, dtype=dt, device=dev)
        self._permute(x, ws, send_buf, send_buf.shape[0], G=G, cum_split=cum_split, dest_base=send_base)
        recv_buf = torch.empty(max(recv_total, 1), d, dtype=dt, device=dev)
        exchange_chunks(S, lay, rank, send_buf, recv_buf, self.group)
        cap = recv_buf.shape[0]
        h = torch.empty(cap, self.experts.ip, dtype=dt, device=dev)
        y = torch.empty(cap, d, dtype=dt, device=dev)
        if ng == 0:
            # no routed rows here: one empty group keeps the launch uniform (shared expert still runs)
            group_offsets = torch.zeros(2, dtype=torch.int32, device=dev)
            group_expert = torch.zeros(1, dtype=torch.int32, device=dev)
            ng = 1
        self._ffn(x, ws, recv_buf, h, y, cap, ng, group_offsets, group_expert)
        ret_buf = torch.empty(max(send_total, 1), d, dtype=dt, device=dev)
        exchange_chunks(S, lay, rank, ret_buf, y, self.group, reverse=True)
        self._combine(ws, ret_buf, ret_buf.shape[0])
        return ws

    def check(self):
        """Synchronise and raise if a kernel recorded an error."""
        L.check(L.load().dsca_check_error(_ptr(self.err), _stream()), "device error word")

    # -------------------------------------------------------------- CUDA graphs
    def capture(self, x: torch.Tensor) -> "ForwardGraph":
        """Capture one forward on the static input `x` [T, d] as a CUDA graph.  Every launch of a
        forward is stream-ordered with device-side counts and plans (no host synchronisation), so
        a replay re-runs the whole block — router, permute or expert-parallel exchange, grouped
        GEMMs, combine — for whatever `x` holds at replay time, for one host call.  One eager
        forward runs first so that set-up (workspace, symmetric region, kernel attributes) happens
        outside the capture; with more than one rank every rank must capture at the same point
        (the eager forward takes part in the exchange).  The expert-cache path (host-side plan per
        forward) and the NCCL exchange (host-side plan) cannot be captured."""
        if self.cache is not None or (self.world > 1 and self.exchange != "p2p"):
            raise NotImplementedError("only the resident and the fused-exchange paths can be captured")
        if x.dim() != 2 or x.shape[1] != self.d or x.dtype != self.dtype or x.device != self.device \
                or not x.is_contiguous():
            raise ValueError("capture needs a contiguous [T, d] input of the engine's dtype and device")
        self.forward(x)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        markers, self.markers = self.markers, None
        try:
            with torch.cuda.graph(graph):
                res = self.forward(x)
        finally:
            self.markers = markers
        return ForwardGraph(graph, x, res)


class ForwardGraph:
    """A captured MoEEngine.forward: `x` is the static input buffer (write the next batch into it),
    replay() runs the block on the current stream and leaves the results in `result` (out, logits,
    topk_ids, expert_index; overwritten by the next replay)."""

    def __init__(self, graph, x: torch.Tensor, result: dict):
        self.graph, self.x, self.result = graph, x, result

    @property
    def out(self) -> torch.Tensor:
        return self.result["out"]

    def replay(self):
        self.graph.replay()


class HostPipeline:
    """MoEEngine.forward over batches that live in pinned host memory, with the PCIe copies
    overlapped: while batch i computes on the current stream, batch i + 1 is copied in on one copy
    stream and batch i - 1's output is copied out on another.  Every batch still crosses PCIe both
    ways; only the waiting overlaps (two device input buffers, event-ordered reuse).

    graphs=True captures the forward once per input buffer (MoEEngine.capture) and replays it:
    one host call per batch instead of one per kernel, so the host keeps ahead of the GPU even
    when many ranks share the host's cores.  Capture is collective across ranks (see capture)."""

    def __init__(self, engine: "MoEEngine", tokens: int, graphs: bool = False):
        self.eng = engine
        dev = engine.device
        self.x_dev = [torch.zeros(tokens, engine.d, dtype=engine.dtype, device=dev) for _ in range(2)]
        self.h2d = torch.cuda.Stream(device=dev)
        self.d2h = torch.cuda.Stream(device=dev)
        self._copied = [torch.cuda.Event() for _ in range(2)]
        self._consumed = [torch.cuda.Event() for _ in range(2)]
        self._drained = [torch.cuda.Event() for _ in range(2)]
        self._used = [False, False]
        self.graphs = [engine.capture(xb) for xb in self.x_dev] if graphs else None

    def _copy_in(self, i, x_host):
        b = i & 1
        with torch.cuda.stream(self.h2d):
            if self._used[b]:
                self.h2d.wait_event(self._consumed[b])  # the forward that read this buffer is done
            self.x_dev[b].copy_(x_host, non_blocking=True)
            self._copied[b].record(self.h2d)

    def run(self, xs_host, outs_host):
        """Forward every xs_host[i] ([T, d], pinned) into outs_host[i] (pinned).  Asynchronous:
        returns once everything is enqueued; synchronize (or wait on .d2h) before reading."""
        main = torch.cuda.current_stream(self.eng.device)
        n = len(xs_host)
        start = torch.cuda.Event()
        start.record(main)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)
        if n:
            self._copy_in(0, xs_host[0])
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                self._copy_in(i + 1, xs_host[i + 1])
            main.wait_event(self._copied[b])
            if self.graphs is not None:
                if self._used[b]:
                    main.wait_event(self._drained[b])  # this graph's last output has been copied out
                self.graphs[b].replay()
                out = self.graphs[b].out
            else:
                out = self.eng.forward(self.x_dev[b])["out"]
            self._consumed[b].record(main)
            self._used[b] = True
            done = torch.cuda.Event()
            done.record(main)
            self.d2h.wait_event(done)
            with torch.cuda.stream(self.d2h):
                outs_host[i].copy_(out, non_blocking=True)
            if self.graphs is not None:
                self._drained[b].record(self.d2h)
            else:
                out.record_stream(self.d2h)
        end = torch.cuda.Event()
        end.record(self.d2h)
        main.wait_event(end)


def default_expert_to_gpu(E: int, G: int) -> np.ndarray:
    """Contiguous blocks, the first E % G GPUs one expert more (60 on 8 -> 4 x 8 + 4 x 7).
    Equals the reference's naive arange(E) // (E // G) when G divides E
    (src/harmonymoe/scheduler.py:215-222)."""
    base, extra = divmod(E, G)
    e2g = np.zeros(E, np.int32)
    e = 0
    for g in range(G):
        n = base + (1 if g < extra else 0)
        e2g[e:e + n] = g
        e += n
    return e2g
