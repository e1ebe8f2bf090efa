"""Tensor parallelism for the batch-1 latency case: one process per GPU (torch.distributed, NCCL),
the Megatron split of the dense Qwen3 layer over its KV heads.

Rank r of t holds (ShardPlan):
- query heads [r*Hq/t, (r+1)*Hq/t) and KV heads [r*Hkv/t, ...) with their rows of q/k/v_proj, its
  own KV cache [layers, batch, Hkv/t, capacity, 128], and the matching columns of o_proj;
- intermediate columns [r*I/t, (r+1)*I/t) of gate/up_proj (rows) and down_proj (columns);
- a vocabulary shard of the tied LM head, on 32-row boundaries (ranks differ by at most 32 rows).

o_proj and down_proj give each rank an unrounded fp32 part of the [batch, hidden] product; an
all-reduce sums the parts and `ipe_add_partial` applies the residual with the single bf16 rounding
of the unsplit layer, so the math is the unsharded engine's up to fp32 summation order. The LM
head shard writes sampling records with global vocabulary IDs (and the winning logit); an
all-gather of the records lets every rank sample the same token (`ipe_sample_records`), keeping
the ranks in lock step without moving logits.

A decode step runs one of three ways (`allreduce`):
- "fused" (default): the one-kernel decode step (ipe_decode_step) with the exchanges inside it.
  Each row-parallel unit pushes its fp32 sums straight into every rank's receive buffer over
  NVLink; the grid barrier after the phase is also a cross-rank flag exchange; the next phase's
  staging sums the parts in rank order, applies the residual and the RMSNorm. The LM-head
  records go to every rank the same way and every rank samples the same token in the kernel.
- "nvlink": the per-operator kernels with a one-shot all-reduce kernel over peer memory.
- "nccl": the per-operator kernels with NCCL all-reduces and an all-gather of the records.
The two per-operator modes are captured once in a CUDA graph, as is the fused step.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ipe_b200 import _native as nat
from ipe_b200.config import check_supported
from ipe_b200.model import decode_tiles, rotary_rows

HEAD_DIM = 128


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    q_heads: int      # local query heads
    kv_heads: int     # local KV heads
    q0: int           # first global query head
    kv0: int          # first global KV head
    inter: int        # local intermediate columns
    i0: int           # first global intermediate column
    vocab_rows: int   # local LM-head rows
    vocab_offset: int  # first global vocabulary ID (a multiple of 32)
    parts: int        # local sampling records per row (vocab_rows / 32, rounded up)
    parts_max: int    # the largest `parts` over the ranks (the all-gather's padded size)


def shard_plan(config, rank: int, world: int) -> ShardPlan:
    """The rows and columns rank `rank` of `world` owns; ValueError if the model does not split."""
    c = config
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if c.num_key_value_heads % world:
        raise ValueError(f"{c.num_key_value_heads} KV heads do not split over {world} ranks")
    if c.intermediate_size % (world * nat.GATE_UP_GROUP):
        raise ValueError(f"intermediate {c.intermediate_size} does not split over {world} ranks in groups of "
                         f"{nat.GATE_UP_GROUP}")
    group = c.num_attention_heads // c.num_key_value_heads
    kv = c.num_key_value_heads // world
    inter = c.intermediate_size // world
    blocks = (c.vocab_size + 31) // 32
    per, extra = divmod(blocks, world)
    first = rank * per + min(rank, extra)
    mine = per + (1 if rank < extra else 0)
    offset = 32 * first
    rows = min(32 * mine, c.vocab_size - offset)
    return ShardPlan(rank, world, kv * group, kv, rank * kv * group, rank * kv, inter, rank * inter, rows, offset,
                     (rows + 31) // 32, per + (1 if extra else 0))


def shard_layer(layer, plan: ShardPlan) -> dict[str, torch.Tensor]:
    """This rank's pieces of one layer's weights (views sliced from the full tensors, made
    contiguous): w_qkv rows, w_o columns, gate / up rows, down columns, and the norms."""
    hd = HEAD_DIM
    q = layer.q_proj[plan.q0 * hd:(plan.q0 + plan.q_heads) * hd]
    k = layer.k_proj[plan.kv0 * hd:(plan.kv0 + plan.kv_heads) * hd]
    v = layer.v_proj[plan.kv0 * hd:(plan.kv0 + plan.kv_heads) * hd]
    cols = slice(plan.i0, plan.i0 + plan.inter)
    return {"w_qkv": torch.cat((q, k, v), 0).contiguous(),
            "w_o": layer.o_proj[:, plan.q0 * hd:(plan.q0 + plan.q_heads) * hd].contiguous(),
            "gate": layer.gate_proj[cols].contiguous(), "up": layer.up_proj[cols].contiguous(),
            "w_down": layer.down_proj[:, cols].contiguous(),
            "in_norm": layer.input_layernorm.contiguous(), "post_norm": layer.post_attention_layernorm.contiguous(),
            "q_norm": layer.q_norm.contiguous(), "k_norm": layer.k_norm.contiguous()}


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Gate and up rows interleaved in groups of IPE_GATE_UP_GROUP (the prefill SiLU*up layout)."""
    g = nat.GATE_UP_GROUP
    rows, k = gate.shape
    return torch.stack((gate.view(rows // g, g, k), up.view(rows // g, g, k)), 1).reshape(2 * rows, k).contiguous()


class _Layer:
    def __init__(self, layer, plan: ShardPlan):
        w = shard_layer(layer, plan)
        self.in_norm, self.post_norm, self.q_norm, self.k_norm = w["in_norm"], w["post_norm"], w["q_norm"], w["k_norm"]
        self.w_qkv, self.w_o, self.w_down = w["w_qkv"], w["w_o"], w["w_down"]
        self.w_gate_up = interleave_gate_up(w["gate"], w["up"])
        self.t_qkv, self.t_o, self.t_down = decode_tiles(self.w_qkv), decode_tiles(self.w_o), decode_tiles(self.w_down)
        self.t_gate_up = decode_tiles(w["gate"], w["up"])


class PeerAllReduce:
    """The group's IPC-mapped communication regions and the fused one-shot all-reduce + residual
    add over NVLink peer memory (ipe_allreduce_residual). Every rank of `group` constructs it (a
    collective), and must `close()` it before the group is destroyed."""

    def __init__(self, group, device: torch.device, slot_bytes: int, region_bytes: int | None = None):
        """slot_bytes: the largest part one all-reduce moves. region_bytes: allocate a region of
        this size instead (the fused decode step's layout, ipe_decode_step_comm_bytes)."""
        import ctypes

        lib = nat.load()
        self.group, self.world, self.rank = group, dist.get_world_size(group), dist.get_rank(group)
        self.slot_bytes = int(slot_bytes)
        size = int(region_bytes) if region_bytes is not None else int(lib.ipe_comm_bytes(self.slot_bytes))
        region = ctypes.c_void_p()
        nat.check(lib.ipe_comm_alloc(size, ctypes.byref(region)), "ipe_comm_alloc")
        self.region = region.value
        handle = (ctypes.c_char * 64)()
        nat.check(lib.ipe_ipc_handle(self.region, handle), "ipe_ipc_handle")
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        pointers, self._opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                pointers.append(self.region)
                continue
            peer = ctypes.c_void_p()
            nat.check(lib.ipe_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(peer)), "ipe_ipc_open")
            pointers.append(peer.value)
            self._opened.append(peer.value)
        self.table = torch.tensor(pointers, dtype=torch.int64, device=device)
        self._slots = [self.region + int(lib.ipe_comm_slot_offset(s, self.slot_bytes)) for s in (0, 1)]

    def slot(self, index: int) -> int:
        """Device address of this rank's slot `index` (where a layer's partial product goes)."""
        return self._slots[index]

    def reduce_residual(self, x: torch.Tensor, count: int, slot: int, stream: int) -> None:
        nat.check(nat.load().ipe_allreduce_residual(x.data_ptr(), count, self.table.data_ptr(), self.world, self.rank,
                                                    slot, self.slot_bytes, stream), "ipe_allreduce_residual")

    def close(self) -> None:
        if self.region is None:
            return
        lib = nat.load()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no peer still reads this rank's region
        for peer in self._opened:
            nat.check(lib.ipe_ipc_close(peer), "ipe_ipc_close")
        dist.barrier(group=self.group)
        nat.check(lib.ipe_comm_free(self.region), "ipe_comm_free")
        self.region, self._opened = None, []


class TensorParallelEngine:
    """prefill / decode / generate of one batch (1..16 rows) with the model split over the ranks of
    `group` (every rank constructs it with the same arguments and calls the same methods in the
    same order). The weights in `loaded` must be bf16 on this rank's GPU; only this rank's shard is
    kept (plus the embedding and the norms, replicated)."""

    def __init__(self, loaded, *, batch: int, capacity: int, group=None, allreduce: str = "fused",
                 wait_limit_s: float = 2.0):
        """wait_limit_s bounds every wait of the one-kernel step on the device, a peer's parts among
        them: a peer that stops answering makes this rank's step give up after that long, set
        device error 3 and commit nothing; `generate` then raises."""
        c, w = loaded.config, loaded.weights
        check_supported(c)
        if w.embed_tokens.dtype != torch.bfloat16 or w.embed_tokens.device.type != "cuda":
            raise ValueError("TensorParallelEngine: bf16 weights on a CUDA device")
        if not (type(batch) is int and 1 <= batch <= 16):
            raise ValueError(f"batch {batch!r}: expected 1..16")
        if not (type(capacity) is int and 1 <= capacity <= c.max_position_embeddings):
            raise ValueError(f"capacity {capacity!r}")
        if not (isinstance(wait_limit_s, (int, float)) and 0 < wait_limit_s <= 60):
            raise ValueError(f"wait_limit_s {wait_limit_s!r}: expected a number of seconds in (0, 60]")
        self.wait_limit_ns = int(wait_limit_s * 1e9)
        self.failed: str | None = None  # set once a step failed on the device; the engine is then spent
        self.group = group
        self.world = dist.get_world_size(group)
        self.plan = p = shard_plan(c, dist.get_rank(group), self.world)
        self.loaded, self.config, self.capacity, self.max_batch = loaded, c, capacity, batch
        self.device = dev = w.embed_tokens.device
        with torch.no_grad():
            self.layers = [_Layer(layer, p) for layer in w.layers]
            self.embed = w.embed_tokens.contiguous()
            self.final_norm = w.norm.contiguous()
            self.t_lm = decode_tiles(w.lm_head[p.vocab_offset:p.vocab_offset + p.vocab_rows].contiguous())
        shape = (c.num_hidden_layers, batch, p.kv_heads, capacity, HEAD_DIM)
        self._k = torch.full(shape, float("nan"), dtype=torch.bfloat16, device=dev)
        self._v = torch.full(shape, float("nan"), dtype=torch.bfloat16, device=dev)
        rows = [rotary_rows(torch.tensor([pos]), c.head_dim, c.rope_theta) for pos in range(capacity)]
        self._cos = torch.cat([r[0] for r in rows]).to(dev).contiguous()
        self._sin = torch.cat([r[1] for r in rows]).to(dev).contiguous()
        lib = nat.load()
        bf, f32 = torch.bfloat16, torch.float32
        self.q_rows = p.q_heads * HEAD_DIM
        self.qkv_rows = (p.q_heads + 2 * p.kv_heads) * HEAD_DIM
        self.x = torch.empty((batch, c.hidden_size), dtype=bf, device=dev)
        self.qkv = torch.empty((batch, self.qkv_rows), dtype=bf, device=dev)
        self.attn = torch.empty((batch, self.q_rows), dtype=bf, device=dev)
        self.act = torch.empty((batch, p.inter), dtype=bf, device=dev)
        self.part = torch.empty((batch, c.hidden_size), dtype=f32, device=dev)
        self.logits = torch.empty((batch, p.vocab_rows), dtype=f32, device=dev)
        # sampling records [parts][rows] (flat), padded to parts_max per rank with neutral records
        self.partials = torch.empty(p.parts_max * batch * nat.PARTIAL_WORDS, dtype=f32, device=dev)
        self.gathered = torch.empty(self.world * p.parts_max * batch * nat.PARTIAL_WORDS, dtype=f32, device=dev)
        self._neutral_records()
        self.state = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device=dev)
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.history_tokens = torch.zeros((batch, capacity), dtype=torch.int64, device=dev)
        self.history_logprobs = torch.zeros((batch, capacity), dtype=f32, device=dev)
        ws = int(lib.ipe_decode_attention_qkv_workspace(batch, p.q_heads, p.kv_heads, capacity))
        self.attn_ws = torch.zeros(ws, dtype=torch.uint8, device=dev)
        linear = max(int(lib.ipe_decode_linear_workspace(batch, r, k)) for r, k in (
            (self.qkv_rows, c.hidden_size), (c.hidden_size, self.q_rows), (2 * p.inter, c.hidden_size),
            (c.hidden_size, p.inter)))
        self.linear_ws = torch.zeros(max(linear, 256), dtype=torch.uint8, device=dev)
        self._prefill: dict[tuple[int, int], dict[str, torch.Tensor]] = {}
        self._graph: torch.cuda.CUDAGraph | None = None
        self._warm = False
        self.batch = 0
        self.length = 0
        if allreduce not in ("fused", "nvlink", "nccl"):
            raise ValueError(f"allreduce {allreduce!r}: expected 'fused', 'nvlink' or 'nccl'")
        # the decode step's all-reduces: inside the one-kernel decode step ("fused"), one-shot kernels
        # over NVLink peer memory ("nvlink"), or NCCL
        self.allreduce = allreduce
        self._peer = None
        if allreduce == "nvlink":
            self._peer = PeerAllReduce(group, dev, batch * c.hidden_size * 4)
        elif allreduce == "fused":
            region = int(lib.ipe_decode_step_comm_bytes(self.world, batch, c.hidden_size))
            self._peer = PeerAllReduce(group, dev, 0, region_bytes=region)
            self.x_alt = torch.empty_like(self.x)
            self.step_ws = torch.zeros(int(lib.ipe_decode_step_workspace(batch, p.q_heads, p.kv_heads, capacity)),
                                       dtype=torch.uint8, device=dev)
            self._layer_descs = self._make_layer_descs()
            self._descs: dict[tuple[int, bool], nat.StepDesc] = {}

    def close(self) -> None:
        """Release the captured step and the peer-memory regions (a collective: every rank calls it
        before the process group is destroyed)."""
        self._graph = None
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    # ------------------------------------------------------------------------ one-kernel step

    def _make_layer_descs(self) -> torch.Tensor:
        """The device array of ipe_layer_desc over this rank's shard tiles and KV cache."""
        import ctypes

        descs = (nat.LayerDesc * len(self.layers))()
        for i, layer in enumerate(self.layers):
            fields = tuple(t.data_ptr() for t in (layer.in_norm, layer.post_norm, layer.q_norm, layer.k_norm,
                                                  layer.t_qkv, layer.t_o, layer.t_gate_up, layer.t_down,
                                                  self._k[i], self._v[i]))
            if any(f % 16 for f in fields):
                raise ValueError(f"layer {i}: the decode step needs 16-byte aligned operands")
            descs[i] = nat.LayerDesc(*fields)
        raw = torch.frombuffer(bytearray(ctypes.string_at(ctypes.addressof(descs), ctypes.sizeof(descs))),
                               dtype=torch.uint8)
        return raw.to(self.device)

    def _step_desc(self, sample: bool) -> nat.StepDesc:
        """ipe_decode_step_desc of this rank's shard: the decode step with its row-parallel sums and
        the LM-head records exchanged inside the kernel over the peers' regions."""
        key = (self.batch, sample)
        d = self._descs.get(key)
        if d is not None:
            return d
        c, p = self.config, self.plan
        d = nat.StepDesc()
        d.layers, d.hidden, d.intermediate = c.num_hidden_layers, c.hidden_size, p.inter
        d.q_heads, d.kv_heads, d.vocab, d.capacity, d.batch = p.q_heads, p.kv_heads, p.vocab_rows, self.capacity, self.batch
        d.eps = c.rms_norm_eps
        d.layer_descs = self._layer_descs.data_ptr()
        d.embed, d.lm_head_tiles, d.final_norm = self.embed.data_ptr(), self.t_lm.data_ptr(), self.final_norm.data_ptr()
        d.cos_table, d.sin_table = self._cos.data_ptr(), self._sin.data_ptr()
        d.state, d.tokens = self.state.data_ptr(), self.tokens.data_ptr()
        d.x, d.qkv, d.attn, d.act = self.x.data_ptr(), self.qkv.data_ptr(), self.attn.data_ptr(), self.act.data_ptr()
        d.logits, d.partials = self.logits.data_ptr(), self.partials.data_ptr()
        d.workspace, d.workspace_bytes = self.step_ws.data_ptr(), self.step_ws.numel()
        if sample:
            d.history_tokens, d.history_logprobs = self.history_tokens.data_ptr(), self.history_logprobs.data_ptr()
            d.history_stride = self.history_tokens.shape[1]
        d.tp_world, d.tp_rank, d.tp_peers = self.world, p.rank, self._peer.table.data_ptr()
        d.x_alt, d.vocab_offset, d.vocab_total = self.x_alt.data_ptr(), p.vocab_offset, c.vocab_size
        d.wait_limit_ns = self.wait_limit_ns
        self._descs[key] = d
        return d

    # ----------------------------------------------------------------------------- collectives

    def _all_reduce(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, group=self.group)

    def _neutral_records(self) -> None:
        """Every record neutral (max and Gumbel max -inf): the padding past a rank's own records."""
        view = self.partials.view(-1, nat.PARTIAL_WORDS)
        view.zero_()
        view[:, 0] = float("-inf")
        view[:, 2] = float("-inf")

    def _gather_records(self) -> None:
        """parts_max records per rank for the live rows, concatenated in rank order."""
        n = self.plan.parts_max * self.batch * nat.PARTIAL_WORDS
        dist.all_gather_into_tensor(self.gathered[:self.world * n], self.partials[:n], group=self.group)

    # ----------------------------------------------------------------------------------- prefill

    def _prefill_buffers(self, batch: int, length: int) -> dict[str, torch.Tensor]:
        key = (batch, length)
        if key not in self._prefill:
            if len(self._prefill) > 4:
                self._prefill.clear()
            c, dev, m = self.config, self.device, batch * length
            bf = torch.bfloat16
            self._prefill[key] = {
                "ids": torch.empty(m, dtype=torch.int64, device=dev),
                "x": torch.empty((m, c.hidden_size), dtype=bf, device=dev),
                "h": torch.empty((m, c.hidden_size), dtype=bf, device=dev),
                "qkv": torch.empty((m, self.qkv_rows), dtype=bf, device=dev),
                "q": torch.empty((batch, self.plan.q_heads, length, HEAD_DIM), dtype=bf, device=dev),
                "attn": torch.empty((m, self.q_rows), dtype=bf, device=dev),
                "act": torch.empty((m, self.plan.inter), dtype=bf, device=dev),
                "part": torch.empty((m, c.hidden_size), dtype=torch.float32, device=dev),
                "cos": None, "sin": None}
            cos, sin = rotary_rows(torch.arange(length), c.head_dim, c.rope_theta)
            self._prefill[key]["cos"], self._prefill[key]["sin"] = cos.to(dev).contiguous(), sin.to(dev).contiguous()
        return self._prefill[key]

    def prefill(self, token_ids: torch.Tensor) -> torch.Tensor:
        """Prompts [B, P] (the same on every rank); fp32 logits [B, V] of the last position."""
        from ipe_b200.forward import check_token_ids

        batch, length = check_token_ids(self.config, token_ids, self.capacity)
        if batch > self.max_batch:
            raise ValueError(f"token_ids: batch {batch} exceeds the {self.max_batch} allocated rows")
        self._set_batch(batch)
        self._run_prefill(token_ids, batch, length)
        self.batch, self.length = batch, length
        return self._full_logits(batch)

    def _run_prefill(self, token_ids: torch.Tensor, batch: int, length: int) -> None:
        c, p, lib = self.config, self.plan, nat.load()
        stream = torch.cuda.current_stream().cuda_stream
        buf = self._prefill_buffers(batch, length)
        m, h, eps = batch * length, c.hidden_size, c.rms_norm_eps
        buf["ids"].copy_(token_ids.reshape(-1).to(torch.int64))
        x = buf["x"]
        nat.check(lib.ipe_embed(buf["ids"].data_ptr(), m, self.embed.data_ptr(), c.vocab_size, h, x.data_ptr(), stream),
                  "ipe_embed")
        for index, layer in enumerate(self.layers):
            nat.check(lib.ipe_rmsnorm(x.data_ptr(), layer.in_norm.data_ptr(), buf["h"].data_ptr(), m, h, eps, 0,
                                      stream), "ipe_rmsnorm")
            nat.check(lib.ipe_gemm(buf["h"].data_ptr(), layer.w_qkv.data_ptr(), buf["qkv"].data_ptr(), m,
                                   self.qkv_rows, h, nat.EPI_STORE, None, stream), "ipe_gemm qkv")
            nat.check(lib.ipe_qk_norm_rope_append(buf["qkv"].data_ptr(), batch, length, p.q_heads, p.kv_heads,
                                                  layer.q_norm.data_ptr(), layer.k_norm.data_ptr(),
                                                  buf["cos"].data_ptr(), buf["sin"].data_ptr(), 0, None,
                                                  buf["q"].data_ptr(), self._k[index].data_ptr(),
                                                  self._v[index].data_ptr(), self.capacity, eps, stream),
                      "ipe_qk_norm_rope_append")
            nat.check(lib.ipe_prefill_attention(buf["q"].data_ptr(), self._k[index].data_ptr(),
                                                self._v[index].data_ptr(), buf["attn"].data_ptr(), batch, p.q_heads,
                                                p.kv_heads, length, self.capacity, stream), "ipe_prefill_attention")
            nat.check(lib.ipe_gemm(buf["attn"].data_ptr(), layer.w_o.data_ptr(), buf["part"].data_ptr(), m, h,
                                   self.q_rows, nat.EPI_PARTIAL, None, stream), "ipe_gemm o_proj")
            self._all_reduce(buf["part"])
            nat.check(lib.ipe_add_partial(x.data_ptr(), buf["part"].data_ptr(), m * h, stream), "ipe_add_partial")
            nat.check(lib.ipe_rmsnorm(x.data_ptr(), layer.post_norm.data_ptr(), buf["h"].data_ptr(), m, h, eps, 0,
                                      stream), "ipe_rmsnorm")
            nat.check(lib.ipe_gemm(buf["h"].data_ptr(), layer.w_gate_up.data_ptr(), buf["act"].data_ptr(), m,
                                   2 * p.inter, h, nat.EPI_SILU_MUL, None, stream), "ipe_gemm gate_up")
            nat.check(lib.ipe_gemm(buf["act"].data_ptr(), layer.w_down.data_ptr(), buf["part"].data_ptr(), m, h,
                                   p.inter, nat.EPI_PARTIAL, None, stream), "ipe_gemm down_proj")
            self._all_reduce(buf["part"])
            nat.check(lib.ipe_add_partial(x.data_ptr(), buf["part"].data_ptr(), m * h, stream), "ipe_add_partial")
        last = x.data_ptr() + (length - 1) * h * 2
        self._lm_head(last, length * h, batch, stream)
        nat.check(lib.ipe_state_set(self.state.data_ptr(), nat.STATE_POS, length, stream), "ipe_state_set")

    def _set_batch(self, batch: int) -> None:
        """A new live batch size: records of the old one must not leak into the padding, and the
        captured step was for the old size."""
        if batch != self.batch:
            self._neutral_records()
            self._graph = None
            self._warm = False
        self.batch = batch

    def _lm_head(self, x_ptr: int, stride: int, batch: int, stream: int) -> None:
        c, p, lib = self.config, self.plan, nat.load()
        nat.check(lib.ipe_lm_head_shard(x_ptr, stride, self.final_norm.data_ptr(), self.t_lm.data_ptr(),
                                        self.logits.data_ptr(), self.partials.data_ptr(), batch, c.hidden_size,
                                        p.vocab_rows, p.vocab_offset, c.rms_norm_eps, 0.0, 0, self.state.data_ptr(),
                                        stream), "ipe_lm_head_shard")

    def _full_logits(self, batch: int) -> torch.Tensor:
        """The [batch, V] fp32 logits of the last step (all ranks' shards gathered)."""
        p = self.plan
        pad = 32 * p.parts_max
        mine = torch.zeros((batch, pad), dtype=torch.float32, device=self.device)
        mine[:, :p.vocab_rows] = self.logits[:batch]
        every = torch.empty((self.world, batch, pad), dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=self.group)
        plans = [shard_plan(self.config, r, self.world) for r in range(self.world)]
        return torch.cat([every[r, :, :q.vocab_rows] for r, q in enumerate(plans)], dim=1)

    # ------------------------------------------------------------------------------------ decode

    def _launch_step(self, sample: bool, stream: int) -> None:
        """One decode step at state[POS] for the rows in self.tokens; with `sample`, the next token
        goes to the history at state[STEP] and to self.tokens, and STEP advances."""
        c, p, lib = self.config, self.plan, nat.load()
        if self.allreduce == "fused":
            import ctypes

            nat.check(lib.ipe_decode_step(ctypes.addressof(self._step_desc(sample)), stream), "ipe_decode_step")
            return
        b, h, eps, st = self.batch, c.hidden_size, c.rms_norm_eps, self.state.data_ptr()
        lws, lwn = self.linear_ws.data_ptr(), self.linear_ws.numel()
        nat.check(lib.ipe_embed(self.tokens.data_ptr(), b, self.embed.data_ptr(), c.vocab_size, h, self.x.data_ptr(),
                                stream), "ipe_embed")
        for index, layer in enumerate(self.layers):
            nat.check(lib.ipe_rmsnorm_qkv(self.x.data_ptr(), layer.in_norm.data_ptr(), layer.t_qkv.data_ptr(),
                                          self.qkv.data_ptr(), b, h, self.qkv_rows, eps, lws, lwn, stream),
                      "ipe_rmsnorm_qkv")
            nat.check(lib.ipe_decode_attention_qkv(self.qkv.data_ptr(), layer.q_norm.data_ptr(),
                                                   layer.k_norm.data_ptr(), self._cos.data_ptr(),
                                                   self._sin.data_ptr(), 0, st, self._k[index].data_ptr(),
                                                   self._v[index].data_ptr(), self.attn.data_ptr(), b, p.q_heads,
                                                   p.kv_heads, self.capacity, eps, self.attn_ws.data_ptr(),
                                                   self.attn_ws.numel(), stream), "ipe_decode_attention_qkv")
            self._row_parallel(lib.ipe_linear_partial, self.attn.data_ptr(), layer.t_o.data_ptr(), self.q_rows, 0,
                               stream)
            nat.check(lib.ipe_rmsnorm_gate_up_silu(self.x.data_ptr(), layer.post_norm.data_ptr(),
                                                   layer.t_gate_up.data_ptr(), self.act.data_ptr(), b, h, p.inter,
                                                   eps, lws, lwn, stream), "ipe_rmsnorm_gate_up_silu")
            self._row_parallel(lib.ipe_linear_partial, self.act.data_ptr(), layer.t_down.data_ptr(), p.inter, 1,
                               stream)
        self._lm_head(self.x.data_ptr(), h, b, stream)
        if sample:
            self._sample(stream)
        nat.check(lib.ipe_state_add(st, nat.STATE_POS, 1, stream), "ipe_state_add")

    def _row_parallel(self, partial, a_ptr: int, tiles_ptr: int, k: int, slot: int, stream: int) -> None:
        """x += this layer's product: each rank's fp32 part (its columns of the weight), summed over
        the ranks, rounded once, added to the residual. slot alternates 0 / 1 between calls."""
        b, h = self.batch, self.config.hidden_size
        lws, lwn = self.linear_ws.data_ptr(), self.linear_ws.numel()
        out = self._peer.slot(slot) if self._peer is not None else self.part.data_ptr()
        nat.check(partial(a_ptr, tiles_ptr, out, b, k, h, lws, lwn, stream), "ipe_linear_partial")
        if self._peer is not None:
            self._peer.reduce_residual(self.x, b * h, slot, stream)
        else:
            self._all_reduce(self.part[:b])
            nat.check(nat.load().ipe_add_partial(self.x.data_ptr(), self.part.data_ptr(), b * h, stream),
                      "ipe_add_partial")

    def _sample(self, stream: int) -> None:
        """Every rank merges every rank's records: the same token on all ranks."""
        self._gather_records()
        b = self.batch
        nat.check(nat.load().ipe_sample_records(self.gathered.data_ptr(), self.world * self.plan.parts_max, b, 0.0,
                                                self.state.data_ptr(), self.history_tokens.data_ptr(),
                                                self.history_logprobs.data_ptr(), self.history_tokens.stride(0),
                                                self.tokens.data_ptr(), stream), "ipe_sample_records")

    def decode(self, tokens: torch.Tensor) -> torch.Tensor:
        """One token per row at position `length`; fp32 logits [B, V] (gathered over the ranks)."""
        if self.batch == 0:
            raise ValueError("decode: no batch; call prefill first")
        if self.length == self.capacity:
            raise ValueError(f"decode: all {self.capacity} positions are committed")
        if self.failed:
            raise RuntimeError(f"tensor-parallel engine: an earlier step failed ({self.failed}); build a new engine")
        if not isinstance(tokens, torch.Tensor) or tokens.shape != (self.batch,):
            raise ValueError(f"tokens: expected integer IDs of shape [{self.batch}]")
        stream = torch.cuda.current_stream().cuda_stream
        nat.check(nat.load().ipe_state_set(self.state.data_ptr(), nat.STATE_POS, self.length, stream), "ipe_state_set")
        self.tokens[:self.batch].copy_(tokens.to(torch.int64))
        self._launch_step(False, stream)
        self.length += 1
        return self._full_logits(self.batch)

    def _step_graph(self) -> None:
        """A sampling decode step: eager the first time, then replayed from a CUDA graph."""
        stream = torch.cuda.current_stream()
        if not self._warm:
            self._launch_step(True, stream.cuda_stream)
            self._warm = True
            return
        if self._graph is None:
            self._graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._graph):
                self._launch_step(True, torch.cuda.current_stream().cuda_stream)
        self._graph.replay()

    def generate(self, token_ids: torch.Tensor, max_new_tokens: int, *, temperature: float = 0.0,
                 seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        """Greedy (temperature 0) or Gumbel-max generation of max_new_tokens per prompt: host
        (tokens [B, N], logprobs [B, N]), identical on every rank."""
        import struct

        from ipe_b200.forward import check_token_ids

        batch, length = check_token_ids(self.config, token_ids, self.capacity)
        if length + max_new_tokens - 1 > self.capacity:
            raise ValueError("prompt length + max_new_tokens - 1 exceeds capacity")
        lib, stream, st = nat.load(), torch.cuda.current_stream().cuda_stream, self.state.data_ptr()
        if batch > self.max_batch:
            raise ValueError(f"token_ids: batch {batch} exceeds the {self.max_batch} allocated rows")
        if self.failed:
            raise RuntimeError(f"tensor-parallel engine: an earlier step failed ({self.failed}); build a new engine")
        nat.device_error(reset=True)  # the check below sees only this call's failures
        nat.check(lib.ipe_state_set(st, nat.STATE_STEP, 0, stream), "ipe_state_set")
        nat.check(lib.ipe_state_set(st, nat.STATE_SEED, int(seed) & (2**63 - 1), stream), "ipe_state_set")
        bits = struct.unpack("<i", struct.pack("<f", float(temperature)))[0]
        nat.check(lib.ipe_state_set(st, nat.STATE_TEMPERATURE, bits, stream), "ipe_state_set")
        try:
            self._set_batch(batch)
            self._run_prefill(token_ids, batch, length)
            self._sample(stream)
            for _ in range(max_new_tokens - 1):
                self._step_graph()
        finally:
            nat.check(lib.ipe_state_set(st, nat.STATE_TEMPERATURE, 0, stream), "ipe_state_set")
        tokens = self.history_tokens[:batch, :max_new_tokens].cpu()
        logprobs = self.history_logprobs[:batch, :max_new_tokens].cpu()
        code = nat.device_error(reset=True)
        if code:
            # a step whose wait ran out (a peer that stopped answering) committed nothing: the
            # device position is the committed prefix, and the exchange epochs are spent
            self.length = int(self.state[nat.STATE_POS].item())
            self.failed = f"device error {code}"
            raise RuntimeError(f"tensor-parallel generate: a decode step failed on the device (error {code}: "
                               f"{'a wait ran out' if code == 3 else 'see ipe_device_error'}); "
                               f"{self.length} positions committed")
        self.length = length + max_new_tokens - 1
        return tokens, logprobs
