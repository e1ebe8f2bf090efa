"""Cached generation for one static batch of equal-length prompts, on the CUDA kernels.

Drop-in for the reference's `ipe.engine` (src/ipe/engine.py): `Engine(loaded, *, batch, capacity,
dtype=None, backend="sdpa")` with `prefill`, `decode`, `generate`, the attributes `batch`,
`length`, `capacity`, `dtype`, `loaded`, the cache tensors `_k` / `_v` ([layers, batch, KV heads,
capacity, head_dim], NaN until written), the rotary rows `_cos` / `_sin`, `_step`, `sample` and
`Generation`, with the reference's argument checks and ValueError messages.

How a step runs: K and V, the rotary rows, every activation buffer and a small device step state
(position, sampled-token index, seed, temperature) are allocated in __init__. A prefill launches
the tensor-core GEMMs, the causal flash-attention and the fused norm/RoPE/append kernel layer by
layer. A decode step reads its position from the device state, so after one eager step it is
captured once into a CUDA graph and replayed; the graph ends by advancing the device position.
`length` (host) advances only after a step's launches succeed, and the device position only at
the end of a step, so a failed step leaves the committed prefix as it was. A decode step
allocates nothing and never reads a device value on the host. One thread, the current stream.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

import torch

from ipe_b200 import _native as nat
from ipe_b200 import fp32 as _fp32
from ipe_b200 import layer as _layer
from ipe_b200 import model as _model
from ipe_b200 import ops
from ipe_b200.forward import INTEGER_DTYPES, check_backend, check_dtype, check_token_ids

# One decoder layer, with the reference's signature (x, layer, rope, config, *, backend, cache=None,
# start=0) (src/ipe/forward.py:86-115). While this module global is the built-in function, steps
# run the engine's fused paths (the one-kernel decode step from a CUDA graph, the fused prefill
# chain). A caller that replaces it (to wrap, count or fail a layer, as the reference's tests do,
# src/ipe/engine.py:107-109) gets it called for every layer of every step, as the reference does.
decoder_layer = _layer.decoder_layer
_BUILTIN_DECODE = _layer.decoder_layer


def _hooked() -> bool:
    return decoder_layer is not _BUILTIN_DECODE


@dataclass(frozen=True, slots=True)
class Generation:
    """Host tensors; n is max_new_tokens unless every sequence stopped earlier."""

    tokens: torch.Tensor  # [B, n] int64
    logprobs: torch.Tensor  # [B, n] fp32: log_softmax of the fp32 logits at each token
    lengths: torch.Tensor  # [B] int64: tokens up to and including the first stop ID, else n


def sample(logits: torch.Tensor, temperature: float,
           generator: torch.Generator | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Tokens [B] and untempered log-probabilities [B] from fp32 logits [B, V] on the GPU.

    Temperature 0: argmax, lowest ID on ties. Otherwise Gumbel-max, argmax(l / T - log(-log U)),
    with U from a counter-based generator keyed by a 64-bit seed taken from `generator` (so the
    same generator seed gives the same draws). No host sync (src/ipe/engine.py:28-41).
    """
    if temperature == 0:
        return ops.sample_logits(logits.contiguous(), 0.0, 0)
    return ops.sample_logits(logits.contiguous(), float(temperature), _generator_seed(generator))


def _mix64(z: int) -> int:
    """splitmix64's finaliser: a 64-bit bijection that spreads every input bit."""
    z &= 2**64 - 1
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & (2**64 - 1)
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & (2**64 - 1)
    return z ^ (z >> 31)


def _generator_seed(generator: torch.Generator | None) -> int:
    """A 64-bit seed from `generator`, advancing it, without reading device memory: a CPU
    generator draws on the host; a CUDA generator's seed and Philox offset are host-side state,
    so the seed mixes the two and the offset moves on by one draw."""
    if generator is None or generator.device.type == "cpu":
        return int(torch.randint(0, 2**62, (1,), generator=generator).item())
    offset = generator.get_offset()
    generator.set_offset(offset + 4)
    return _mix64(generator.initial_seed() ^ _mix64(0x9E3779B97F4A7C15 * (offset // 4 + 1)))


def _step_seed(seed: int, step: int) -> int:
    """A 64-bit seed per generation step for the fp32 path's sampler."""
    return _mix64(seed + 0x9E3779B97F4A7C15 * (step + 1))


def _float_bits(value: float) -> int:
    return struct.unpack("<i", struct.pack("<f", float(value)))[0]


class Engine:
    """Prefill, decode and generate over a KV cache of batch rows and capacity positions."""

    def __init__(self, loaded, *, batch: int, capacity: int, dtype: torch.dtype | None = None,
                 backend: str = "sdpa"):
        config = loaded.config
        dtype = loaded.weights.embed_tokens.dtype if dtype is None else dtype
        check_dtype(loaded, dtype, (torch.bfloat16, torch.float32))
        check_backend(backend)
        if type(batch) is not int or batch < 1:
            raise ValueError(f"batch {batch!r}: expected an integer >= 1")
        if batch > 16:
            raise ValueError(f"batch {batch}: the decode kernels take at most 16 rows")
        if type(capacity) is not int or not 1 <= capacity <= config.max_position_embeddings:
            raise ValueError(f"capacity {capacity!r}: expected an integer from 1 to {config.max_position_embeddings}")
        self.loaded, self.dtype, self.backend, self.capacity = loaded, dtype, backend, capacity
        self.batch = 0
        self.length = 0
        self._f32 = None
        if dtype == torch.float32:
            # the fp32 path: reference-precision kernels, one launch per operator (ipe_b200.fp32)
            self._f32 = _fp32.fp32_model(loaded)
            shape = (config.num_hidden_layers, batch, config.num_key_value_heads, capacity, config.head_dim)
            self._k = torch.full(shape, float("nan"), dtype=dtype, device=self._f32.device)
            self._v = torch.full(shape, float("nan"), dtype=dtype, device=self._f32.device)
            self._cos, self._sin = self._f32.decode_rotary(capacity)
            self._f32_buffers: dict[tuple[int, int], _fp32.Fp32Buffers] = {}
            return
        self._model = _model.packed_model(loaded)
        device = self._model.device
        shape = (config.num_hidden_layers, batch, config.num_key_value_heads, capacity, config.head_dim)
        self._k = torch.full(shape, float("nan"), dtype=dtype, device=device)
        self._v = torch.full(shape, float("nan"), dtype=dtype, device=device)
        self._cos, self._sin = self._model.decode_rotary(capacity)
        self._buf = _model.DecodeBuffers(self._model, batch, capacity)
        self._layer_descs = _model.layer_descs(self._model, self._k, self._v)
        self._step_descs: dict[tuple[int, bool], object] = {}
        self._prefill_buf: _model.PrefillBuffers | None = None
        self._graphs: dict[tuple[int, bool], torch.cuda.CUDAGraph] = {}
        self._warm: set[tuple[int, bool]] = set()  # step variants already run once outside capture
        self._device_pos = 0  # what state[POS] holds once the queued work has run

    # ------------------------------------------------------------------------------- public API

    def prefill(self, token_ids: torch.Tensor) -> torch.Tensor:
        """Start a new batch from prompts [B, P]; fp32 logits [B, V] at position P-1."""
        batch, length = check_token_ids(self.loaded.config, token_ids, self.capacity)
        if batch > self._k.shape[1]:
            raise ValueError(f"token_ids: batch {batch} exceeds the {self._k.shape[1]} allocated rows")
        self.batch = self.length = 0
        cos, sin = (self._f32 or self._model).prefill_rotary(length)
        logits = self._step(token_ids, (cos, sin), 0)
        self.batch, self.length = batch, length
        return logits.clone()

    def decode(self, tokens: torch.Tensor) -> torch.Tensor:
        """One token per sequence [B] at position `length`; fp32 logits [B, V].

        Host IDs are bounds-checked; IDs on the device (the sampler's output) are not, since that
        would sync every step (out-of-range device IDs embed as zeros and set the device error).
        """
        if self.batch == 0:
            raise ValueError("decode: no batch; call prefill first")
        if self.length == self.capacity:
            raise ValueError(f"decode: all {self.capacity} positions are committed")
        if not isinstance(tokens, torch.Tensor) or tokens.shape != (self.batch,) or tokens.dtype not in INTEGER_DTYPES:
            raise ValueError(f"tokens: expected integer IDs of shape [{self.batch}]")
        if tokens.device.type == "cpu":
            check_token_ids(self.loaded.config, tokens[:, None], 1)
        rope = (self._cos[self.length:self.length + 1], self._sin[self.length:self.length + 1])
        logits = self._step(tokens[:, None], rope, self.length)
        self.length += 1
        return logits.clone()

    def generate(self, token_ids: torch.Tensor, max_new_tokens: int, *, temperature: float = 0.0,
                 seed: int = 0, stop_ids: tuple[int, ...] = ()) -> Generation:
        """Generate max_new_tokens per prompt in token_ids [B, P]; needs P + max_new_tokens - 1
        positions. Stops early only when every sequence has emitted a stop ID (one sync per step
        when stop_ids are given)."""
        if type(max_new_tokens) is not int or max_new_tokens < 1:
            raise ValueError(f"max_new_tokens {max_new_tokens!r}: expected an integer >= 1")
        if not (isinstance(temperature, (int, float)) and temperature >= 0):
            raise ValueError(f"temperature {temperature!r}: expected a number >= 0")
        _, length = check_token_ids(self.loaded.config, token_ids, self.capacity)
        if length + max_new_tokens - 1 > self.capacity:
            raise ValueError(f"prompt length {length} + max_new_tokens {max_new_tokens} - 1 exceeds capacity {self.capacity}")
        run = self._generate_stepwise if self._f32 is not None or _hooked() else self._generate_on_device
        tokens, logprobs, lengths, produced = run(token_ids, max_new_tokens, float(temperature), int(seed),
                                                  tuple(stop_ids))
        return Generation(tokens[:, :produced].cpu(), logprobs[:, :produced].cpu(), lengths.cpu())

    def _generate_on_device(self, token_ids, max_new_tokens: int, temperature: float, seed: int,
                            stop_ids: tuple[int, ...] = (), after_prefill=None):
        """The generation loop with its results left on the device: (tokens [B, N], logprobs [B, N],
        lengths [B], produced). `after_prefill()` is called once the prefill is queued (timing hook).

        The first token comes from the fused sampler over the prefill's LM-head records; every later
        one from a decode step that samples its own logits (one kernel per step, replayed from a
        CUDA graph): the sampled ID goes to the history and becomes the next step's input."""
        device = self._model.device
        stream = torch.cuda.current_stream().cuda_stream
        lib, buf = nat.load(), self._buf
        state = buf.state.data_ptr()
        nat.check(lib.ipe_state_set(state, nat.STATE_STEP, 0, stream), "ipe_state_set")
        nat.check(lib.ipe_state_set(state, nat.STATE_SEED, seed & (2**63 - 1), stream), "ipe_state_set")
        nat.check(lib.ipe_state_set(state, nat.STATE_TEMPERATURE, _float_bits(temperature), stream), "ipe_state_set")
        stops = torch.tensor(stop_ids, dtype=torch.int64, device=device) if stop_ids else None
        try:
            self.prefill(token_ids)
            if after_prefill is not None:
                after_prefill()
            batch, vocab = self.batch, self.loaded.config.vocab_size
            tokens, logprobs = buf.history_tokens[:batch], buf.history_logprobs[:batch]
            nat.check(lib.ipe_sample(buf.partials.data_ptr(), buf.logits.data_ptr(), batch, vocab, temperature, state,
                                     tokens.data_ptr(), logprobs.data_ptr(), tokens.stride(0), buf.tokens.data_ptr(),
                                     stream), "ipe_sample")
            lengths = torch.full((batch,), max_new_tokens, dtype=torch.int64, device=device)
            stopped = torch.zeros(batch, dtype=torch.bool, device=device)
            produced = max_new_tokens
            for step in range(max_new_tokens):
                if stops is not None:
                    first = torch.isin(tokens[:, step], stops) & ~stopped
                    lengths = torch.where(first, step + 1, lengths)
                    stopped |= first
                    if bool(stopped.all()):
                        produced = step + 1
                        break
                if step + 1 < max_new_tokens:
                    self._decode_from_buffer(sample=True)
        finally:
            nat.check(lib.ipe_state_set(state, nat.STATE_TEMPERATURE, 0, stream), "ipe_state_set")
        return tokens[:, :max_new_tokens].clone(), logprobs[:, :max_new_tokens].clone(), lengths, produced

    def _generate_stepwise(self, token_ids, max_new_tokens: int, temperature: float, seed: int,
                           stop_ids: tuple[int, ...] = ()):
        """The generation loop of the fp32 path and of a replaced layer hook: prefill, then per
        token the library sampler on the step's fp32 logits (Gumbel draws keyed by a per-step seed)
        and a decode step on the sampled IDs (src/ipe/engine.py:137-147)."""
        logits = self.prefill(token_ids)
        device, batch = self._k.device, self.batch
        tokens = torch.empty((batch, max_new_tokens), dtype=torch.int64, device=device)
        logprobs = torch.empty((batch, max_new_tokens), dtype=torch.float32, device=device)
        stops = torch.tensor(stop_ids, dtype=torch.int64, device=device) if stop_ids else None
        lengths = torch.full((batch,), max_new_tokens, dtype=torch.int64, device=device)
        stopped = torch.zeros(batch, dtype=torch.bool, device=device)
        produced = max_new_tokens
        for step in range(max_new_tokens):
            token, logprob = ops.sample_logits(logits, temperature, _step_seed(seed, step))
            tokens[:, step], logprobs[:, step] = token, logprob
            if stops is not None:
                first = torch.isin(token, stops) & ~stopped
                lengths = torch.where(first, step + 1, lengths)
                stopped |= first
                if bool(stopped.all()):
                    produced = step + 1
                    break
            if step + 1 < max_new_tokens:
                logits = self.decode(token)
        return tokens, logprobs, lengths, produced

    def kernel_launches(self, prompt: int, new_tokens: int) -> dict[str, int]:
        """How many library kernels one `generate(prompt, new_tokens)` launches, by phase."""
        layers = self.loaded.config.num_hidden_layers
        prefill = 1 + layers * 8 + 2  # embed; norm, qkv, rope/append, attention, o, norm, gate/up, down; head, state
        decode = 1  # the whole step, sampling included, is one kernel (plus a 8-byte memset node)
        return {"prefill": prefill, "decode_step": decode, "sample": 1,
                "generate": 4 + prefill + 1 + (new_tokens - 1) * decode}

    # ---------------------------------------------------------------------------------- steps

    def _decode_from_buffer(self, sample: bool = False) -> None:
        """A decode step whose input tokens are already in the device token buffer."""
        if self.length == self.capacity:
            raise ValueError(f"decode: all {self.capacity} positions are committed")
        self._run_decode(self.length, sample=sample)
        self.length += 1

    def _step(self, token_ids: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor], start: int) -> torch.Tensor:
        """Run all layers for token_ids [B, T] at positions start..start+T-1 and the LM head on the
        last position; fp32 logits [B, V] in the engine's logits buffer (src/ipe/engine.py:103-111)."""
        if _hooked():
            return self._step_hooked(token_ids, rope, start)
        if self._f32 is not None:
            return self._step_f32(token_ids, start)
        if start == 0:
            return self._prefill(token_ids, rope)
        if token_ids.shape[1] != 1:
            raise ValueError("decoder_layer: a step after position 0 takes one token; chunked prefill is not supported")
        b = token_ids.shape[0]
        self._buf.tokens[:b].copy_(token_ids[:, 0], non_blocking=True)
        self._run_decode(start, batch=b)
        return self._buf.logits[:b]

    def _step_hooked(self, token_ids: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor], start: int) -> torch.Tensor:
        """The reference's step structure (src/ipe/engine.py:103-111) around a replaced layer hook:
        embedding, the module global `decoder_layer` for every layer with the layer's cache rows,
        then the final norm of each row's last position and the tied LM head, on the CUDA kernels."""
        c, w = self.loaded.config, self.loaded.weights
        batch, length = token_ids.shape
        if start > 0 and length != 1:
            raise ValueError("decoder_layer: a step after position 0 takes one token; chunked prefill is not supported")
        device = self._k.device
        stream = torch.cuda.current_stream().cuda_stream
        lib = nat.load()
        ids = token_ids.to(device=device, dtype=torch.int64).reshape(-1).contiguous()
        x = torch.empty((batch * length, c.hidden_size), dtype=self.dtype, device=device)
        table = self._f32.embed if self._f32 is not None else self._model.embed
        embed = lib.ipe_embed_f32 if self._f32 is not None else lib.ipe_embed
        nat.check(embed(ids.data_ptr(), ids.numel(), table.data_ptr(), c.vocab_size, c.hidden_size, x.data_ptr(),
                        stream), "ipe_embed")
        x = x.view(batch, length, c.hidden_size)
        for index, layer in enumerate(w.layers):
            cache = (self._k[index, :batch], self._v[index, :batch])
            x = decoder_layer(x, layer, rope, c, backend=self.backend, cache=cache, start=start)
        last = x[:, -1].contiguous()
        if self._f32 is not None:
            hidden = _fp32.final_norm(self._f32, last, torch.empty_like(last), stream)
            logits = torch.empty((batch, c.vocab_size), dtype=torch.float32, device=device)
            return _fp32.lm_logits(self._f32, hidden, logits, stream)
        m, buf = self._model, self._buf
        nat.check(lib.ipe_lm_head(last.data_ptr(), c.hidden_size, m.final_norm.data_ptr(), m.t_lm_head.data_ptr(),
                                  buf.logits.data_ptr(), buf.partials.data_ptr(), batch, c.hidden_size, c.vocab_size,
                                  c.rms_norm_eps, 0.0, 0, buf.state.data_ptr(), stream), "ipe_lm_head")
        return buf.logits[:batch]

    def _step_f32(self, token_ids: torch.Tensor, start: int) -> torch.Tensor:
        """The fp32 path of _step: token_ids [B, T] at positions start.., logits of each row's last
        position."""
        batch, tokens = token_ids.shape
        buf = self._f32_buffers.get((batch, tokens))
        if buf is None:
            if len(self._f32_buffers) > 8:
                self._f32_buffers.clear()
            buf = self._f32_buffers[(batch, tokens)] = _fp32.Fp32Buffers(self._f32, batch, tokens)
        buf.ids.copy_(token_ids.reshape(-1), non_blocking=True)
        cos, sin = self._f32.prefill_rotary(tokens) if start == 0 else (self._cos, self._sin)
        stream = torch.cuda.current_stream().cuda_stream
        _fp32.run_layers(self._f32, buf, self._k, self._v, start, self.capacity, cos, sin, stream)
        return _fp32.step_logits(self._f32, buf, stream)

    def _prefill(self, token_ids: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
        c, m = self.loaded.config, self._model
        batch, length = token_ids.shape
        tokens = batch * length
        if self._prefill_buf is None or self._prefill_buf.tokens < tokens or self._prefill_buf.q.shape[2] != length \
                or self._prefill_buf.q.shape[0] != batch:
            self._prefill_buf = None
            self._prefill_buf = _model.PrefillBuffers(m, tokens, batch, length)
        buf = self._prefill_buf
        stream = torch.cuda.current_stream().cuda_stream
        lib = nat.load()
        ids = token_ids.to(device=m.device, dtype=torch.int64).reshape(-1).contiguous()
        nat.check(lib.ipe_embed(ids.data_ptr(), tokens, m.embed.data_ptr(), c.vocab_size, c.hidden_size,
                                buf.x.data_ptr(), stream), "ipe_embed")
        cos, sin = rope
        for index in range(c.num_hidden_layers):
            _model.prefill_layer(m, index, buf, self._k[index], self._v[index], batch, length, self.capacity, cos, sin,
                                 stream)
        last = buf.x.data_ptr() + (length - 1) * c.hidden_size * 2
        nat.check(lib.ipe_lm_head(last, length * c.hidden_size, m.final_norm.data_ptr(), m.t_lm_head.data_ptr(),
                                  self._buf.logits.data_ptr(), self._buf.partials.data_ptr(), batch, c.hidden_size,
                                  c.vocab_size, c.rms_norm_eps, 0.0, 0, self._buf.state.data_ptr(), stream),
                  "ipe_lm_head")
        nat.check(lib.ipe_state_set(self._buf.state.data_ptr(), nat.STATE_POS, length, stream), "ipe_state_set")
        self._device_pos = length
        return self._buf.logits[:batch]

    def _launch_step(self, batch: int, sample: bool, stream: int) -> None:
        """The whole decode step as one kernel (ipe_decode_step)."""
        import ctypes

        key = (batch, sample)
        desc = self._step_descs.get(key)
        if desc is None:
            desc = _model.step_desc(self._model, self._buf, self._layer_descs, batch, self.capacity, self._cos,
                                    self._sin, sample)
            self._step_descs[key] = desc
        nat.check(nat.load().ipe_decode_step(ctypes.addressof(desc), stream), "ipe_decode_step")

    def _run_decode(self, start: int, batch: int | None = None, sample: bool = False) -> None:
        batch = self.batch if batch is None else batch
        stream = torch.cuda.current_stream().cuda_stream
        if self._device_pos != start:
            nat.check(nat.load().ipe_state_set(self._buf.state.data_ptr(), nat.STATE_POS, start, stream),
                      "ipe_state_set")
        if (batch, sample) not in self._warm:
            self._launch_step(batch, sample, stream)
            self._warm.add((batch, sample))
        else:
            graph = self._graphs.get((batch, sample))
            if graph is None:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    self._launch_step(batch, sample, torch.cuda.current_stream().cuda_stream)
                self._graphs[(batch, sample)] = graph
            graph.replay()
        self._device_pos = start + 1
