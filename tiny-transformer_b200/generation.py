"""End-to-end greedy generation with the sm_100a attention (the caller side of the hot path).

A pre-norm decoder with tied embeddings and a contiguous KV cache, restating the reference's
``Transformer`` / ``Block`` / ``KVCache`` (tiny_transformer/model.py:11-136) with its operator
choices reduced to the one this package replaces: ``attention`` is "student" (this package's
kernels), "sdpa" (torch SDPA, reference.py:56-64) or "reference" (the reference's executable
specification, reference.py:49-53); every other operator is the reference's torch expression
(reference.py:16-34, 67-72). Weights are random N(0, 0.02) as in model.py:93-99.

Two decode paths:

* eager (``Decoder.forward`` with a cache): the reference's call sequence. The cache's prefix
  views ``[B, H, :end, D]`` go to the attention operator as they are; the student kernels read
  them in place (row stride = 128 B), where the reference's native path copies the whole
  prefix of every layer at every step (attention.cu:74-76).
* graphed (``GraphedDecode``): one decode step (embedding, all layers, K/V append, attention,
  logits, argmax, position advance) captured once in a CUDA graph.

With the student attention and a cache, RoPE on q/k and the K/V append run as one kernel per
layer reading FP32 cos/sin tables built once per model, in place of the reference's ~20
elementwise launches for ``rope`` and ``KVCache.update``: inside the QKV projection's epilogue
(``operators.fused.qkv_rope_append``, the projection never written to memory) when the width
is a multiple of 64, else after the cuBLAS projection
(``operators.fused.rope_append``). Attention reads the
  full-capacity cache with per-sequence lengths ``kv_lens`` held on the device, so the same
  graph serves every step and the host only replays it.

``request`` measures TTFT / TPOT / tokens per second the way the reference's model benchmark
does (tiny_transformer/benchmarks/model.py:19-37).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

ATTENTION_BACKENDS = ("student", "sdpa", "reference")


@dataclass(frozen=True)
class DecoderConfig:
    """Shape of the decoder; the defaults are configs/model_60m.json of the reference."""
    vocab_size: int = 8192
    dim: int = 768
    n_layers: int = 8
    n_heads: int = 12
    hidden_dim: int = 2048
    max_seq_len: int = 4096
    norm_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads


# ------------------------------------------------------------------------ operators

def _accumulation(x):
    """FP32 for half-precision tensors, unchanged otherwise (reference.py:12-13)."""
    return x.float() if x.dtype in (torch.float16, torch.bfloat16) else x


def rms_norm(x, weight, eps):
    """RMSNorm in FP32 for half-precision inputs, output in the input dtype (reference.py:24-27)."""
    xf = _accumulation(x)
    y = xf * torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps)
    return (y * weight.to(xf.dtype)).to(x.dtype)


def rope(x, cos, sin):
    """Rotary embedding over adjacent pairs (0,1), (2,3), ... (reference.py:30-34)."""
    even, odd = x[..., 0::2], x[..., 1::2]
    cos, sin = cos.to(x.dtype), sin.to(x.dtype)
    return torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1).flatten(-2)


def _causal_allowed(tq, tk, past_len, device):
    q_pos = torch.arange(tq, device=device) + past_len
    k_pos = torch.arange(tk, device=device)
    return (k_pos[None, :] <= q_pos[:, None])[None, None]


def reference_attention(q, k, v, past_len=0):
    """The reference's executable specification (reference.py:49-53), on any device."""
    scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    scores = _accumulation(scores).masked_fill(
        ~_causal_allowed(q.shape[-2], k.shape[-2], past_len, q.device), float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1).to(v.dtype), v)


def sdpa_attention(q, k, v, past_len=0):
    """torch SDPA with the reference's mask alignment rules (reference.py:56-64)."""
    if past_len == 0 and q.shape[-2] == k.shape[-2]:
        return F.scaled_dot_product_attention(q, k, v, is_causal=True)
    if q.shape[-2] == 1:
        return F.scaled_dot_product_attention(q, k, v, is_causal=False)
    mask = _causal_allowed(q.shape[-2], k.shape[-2], past_len, q.device)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask)


def student_attention(q, k, v, past_len=0):
    from .operators import student
    return student.attention(q, k, v, past_len)


def attention_operator(name: str):
    """The attention implementation selected like ``--op attention=<name>`` (dispatch.py:13-17)."""
    table = {"student": student_attention, "sdpa": sdpa_attention,
             "reference": reference_attention}
    if name not in table:
        raise ValueError(f"Unsupported backend {name!r} for attention")
    return table[name]


# ------------------------------------------------------------------------ KV cache

class KVCache:
    """Inference cache with the reference's semantics (model.py:11-43): per-layer storage
    ``[B, H, capacity, D]`` allocated on first use; ``update`` writes the new keys/values at
    ``[length, end)`` and returns the live prefix as views; ``length`` advances once per model
    call, not per layer."""

    def __init__(self, config: DecoderConfig, batch_size: int, capacity: int):
        if not 0 < capacity <= config.max_seq_len or batch_size <= 0:
            raise ValueError("invalid KV cache batch size or capacity")
        self.batch_size = batch_size
        self.capacity = capacity
        self.length = 0
        self.keys = [None] * config.n_layers
        self.values = [None] * config.n_layers

    def reset(self):
        self.length = 0

    def _storage(self, layer, k, v):
        if self.keys[layer] is None:
            shape = (self.batch_size, k.shape[1], self.capacity, k.shape[-1])
            self.keys[layer] = k.new_empty(shape)
            self.values[layer] = v.new_empty(shape)
        elif self.keys[layer].dtype != k.dtype or self.keys[layer].device != k.device:
            raise ValueError("KV cache dtype/device changed; create a new cache")
        return self.keys[layer], self.values[layer]

    def update(self, layer, k, v):
        end = self.length + k.shape[-2]
        if end > self.capacity or k.shape[0] != self.batch_size:
            raise ValueError("KV cache capacity exceeded or batch size changed")
        keys, values = self._storage(layer, k, v)
        keys[:, :, self.length:end, :].copy_(k)
        values[:, :, self.length:end, :].copy_(v)
        return keys[:, :, :end, :], values[:, :, :end, :]

    def storage_for(self, layer, qkv):
        """The layer's [B, H, capacity, D] storage for a [B, T, 3, H, D] projection."""
        b, _, _, h, d = qkv.shape
        if b != self.batch_size:
            raise ValueError("KV cache capacity exceeded or batch size changed")
        proto = qkv.new_empty((b, h, 1, d))
        return self._storage(layer, proto, proto)

    def append_at(self, layer, k, v, position: torch.Tensor):
        """Write one step's keys/values at the device-held ``position`` (int64, shape [1]);
        returns the full-capacity storage. Used inside a captured decode step."""
        keys, values = self._storage(layer, k, v)
        keys.index_copy_(2, position, k)
        values.index_copy_(2, position, v)
        return keys, values

    def allocated_bytes(self):
        return sum(x.numel() * x.element_size() for x in self.keys + self.values if x is not None)


# ------------------------------------------------------------------------ model

class Block(nn.Module):
    """One pre-norm decoder block (model.py:46-76)."""

    def __init__(self, config: DecoderConfig):
        super().__init__()
        self.config = config
        self.attn_norm = nn.Parameter(torch.ones(config.dim))
        self.ffn_norm = nn.Parameter(torch.ones(config.dim))
        self.qkv = nn.Parameter(torch.empty(3 * config.dim, config.dim))
        self.proj = nn.Parameter(torch.empty(config.dim, config.dim))
        self.gate_up = nn.Parameter(torch.empty(2 * config.hidden_dim, config.dim))
        self.down = nn.Parameter(torch.empty(config.dim, config.hidden_dim))

    def project_qkv(self, x, cos, sin):
        cfg = self.config
        batch, time, _ = x.shape
        h = rms_norm(x, self.attn_norm, cfg.norm_eps)
        qkv = F.linear(h, self.qkv).reshape(batch, time, 3, cfg.n_heads, cfg.head_dim)
        q, k, v = (t.transpose(1, 2) for t in qkv.unbind(dim=2))
        return rope(q, cos, sin), rope(k, cos, sin), v

    def finish(self, x, attended):
        cfg = self.config
        batch, _, time, _ = attended.shape
        x = x + F.linear(attended.transpose(1, 2).reshape(batch, time, cfg.dim), self.proj)
        h = rms_norm(x, self.ffn_norm, cfg.norm_eps)
        gate, up = F.linear(h, self.gate_up).chunk(2, dim=-1)
        return x + F.linear(F.silu(gate) * up, self.down)

    def forward(self, x, attention, cos, sin, layer, cache=None):
        q, k, v = self.project_qkv(x, cos, sin)
        past_len = 0 if cache is None else cache.length
        if cache is not None:
            k, v = cache.update(layer, k, v)
        return self.finish(x, attention(q, k, v, past_len))

    def qkv_rows(self, x):
        """The fused QKV projection as a contiguous [B, T, 3, H, 64] tensor."""
        cfg = self.config
        batch, time, _ = x.shape
        h = rms_norm(x, self.attn_norm, cfg.norm_eps)
        return F.linear(h, self.qkv).view(batch, time, 3, cfg.n_heads, cfg.head_dim)

    def forward_fused(self, x, tables, layer, cache, position, kv_lens=None, fused_qkv=False):
        """Student path: one kernel applies RoPE to q/k and appends k/v to the cache
        (operators.fused.rope_append), then attention reads the cache in place. With
        ``fused_qkv`` the QKV projection itself runs in that kernel too (its epilogue applies
        RoPE and writes the cache rows; the projection never reaches memory). With ``kv_lens``
        (captured decode) attention sees the full-capacity cache masked per sequence;
        otherwise the live prefix [0, position + T)."""
        from .operators import fused, student
        cfg = self.config
        if fused_qkv:
            batch = x.shape[0]
            if batch != cache.batch_size:
                raise ValueError("KV cache capacity exceeded or batch size changed")
            h = rms_norm(x, self.attn_norm, cfg.norm_eps).contiguous()
            proto = h.new_empty((batch, cfg.n_heads, 1, cfg.head_dim))
            keys, values = cache._storage(layer, proto, proto)
            q = fused.qkv_rope_append(h, self.qkv, tables[0], tables[1], position, keys, values)
        else:
            qkv = self.qkv_rows(x)
            keys, values = cache.storage_for(layer, qkv)
            q = fused.rope_append(qkv, tables[0], tables[1], position, keys, values)
        if kv_lens is not None:
            attended = student.attention(q, keys, values, cache.capacity - 1, None, kv_lens)
        else:
            end = position + x.shape[1]
            attended = student.attention(q, keys[:, :, :end], values[:, :, :end], position)
        return self.finish(x, attended)


class Decoder(nn.Module):
    """Decoder with tied embeddings (model.py:79-136), attention chosen by name."""

    def __init__(self, config: DecoderConfig, attention: str = "student"):
        super().__init__()
        self.config = config
        self.attention_name = attention
        self.attention = attention_operator(attention)
        self.embedding = nn.Parameter(torch.empty(config.vocab_size, config.dim))
        self.blocks = nn.ModuleList(Block(config) for _ in range(config.n_layers))
        self.final_norm = nn.Parameter(torch.ones(config.dim))
        for parameter in self.parameters():
            if parameter.ndim >= 2:
                nn.init.normal_(parameter, mean=0.0, std=0.02)
        for block in self.blocks:
            for parameter in (block.proj, block.down):
                nn.init.normal_(parameter, std=0.02 / (2 * config.n_layers) ** 0.5)
        # RoPE tables for every position, FP32: the values model.py:114-118 computes per call,
        # computed on the model's device like there (rebuilt whenever the model moves).
        self.register_buffer("rope_cos", torch.empty(0), persistent=False)
        self.register_buffer("rope_sin", torch.empty(0), persistent=False)
        self._build_rope_tables()
        # With the student attention, RoPE + cache append run as one fused kernel, and (when
        # the width is a multiple of 64) inside the QKV projection's epilogue.
        self.fused_rope = True
        self.fused_qkv = config.dim % 64 == 0

    def _build_rope_tables(self):
        positions = torch.arange(self.config.max_seq_len, device=self.embedding.device)
        cos, sin = self.rope_tables(positions)
        self.rope_cos = cos[0, 0].contiguous()
        self.rope_sin = sin[0, 0].contiguous()

    def _apply(self, fn, recurse=True):
        # Moving or casting the model (e.g. .to("cuda", torch.bfloat16)) rebuilds the FP32
        # tables on the new device instead of rounding or copying them.
        out = super()._apply(fn, recurse)
        self._build_rope_tables()
        return out

    def set_attention(self, name: str):
        self.attention_name = name
        self.attention = attention_operator(name)

    def uses_fused(self, cache) -> bool:
        return cache is not None and self.fused_rope and self.attention_name == "student"

    def new_cache(self, batch_size, capacity=None):
        return KVCache(self.config, batch_size,
                       self.config.max_seq_len if capacity is None else capacity)

    def rope_tables(self, positions: torch.Tensor):
        """cos/sin [1, 1, T, D/2] for int positions [T], built in FP32 (model.py:114-118)."""
        d = self.config.head_dim
        freq = 1.0 / self.config.rope_theta ** (
            torch.arange(0, d, 2, device=positions.device).float() / d)
        angles = positions.float()[None, :, None] * freq
        return angles.cos()[:, None], angles.sin()[:, None]

    def logits(self, x):
        x = rms_norm(x, self.final_norm, self.config.norm_eps)
        return F.linear(x, self.embedding)

    def forward(self, ids, cache: KVCache | None = None, last_only=False):
        if ids.ndim != 2 or ids.shape[1] == 0:
            raise ValueError("ids must have shape [batch, nonzero time]")
        past_len = 0 if cache is None else cache.length
        time_ = ids.shape[1]
        if time_ + past_len > self.config.max_seq_len:
            raise ValueError("sequence exceeds model max_seq_len")
        if cache is not None:
            if self.training or torch.is_grad_enabled():
                raise ValueError("KV cache requires eval() and torch.no_grad()/inference_mode()")
            if time_ + past_len > cache.capacity or ids.shape[0] != cache.batch_size:
                raise ValueError("KV cache capacity exceeded or batch size changed")
        x = F.embedding(ids, self.embedding)
        if self.uses_fused(cache):
            tables = (self.rope_cos, self.rope_sin)
            for layer, block in enumerate(self.blocks):
                x = block.forward_fused(x, tables, layer, cache, past_len,
                                        fused_qkv=self.fused_qkv)
        else:
            cos, sin = self.rope_tables(torch.arange(past_len, past_len + time_, device=ids.device))
            for layer, block in enumerate(self.blocks):
                x = block(x, self.attention, cos, sin, layer, cache)
        if cache is not None:
            cache.length += time_
        if last_only:
            x = x[:, -1:, :]
        return self.logits(x)


# ------------------------------------------------------------------------ graphed decode

class GraphedDecode:
    """One greedy decode step of ``model`` over ``cache``, captured once in a CUDA graph.

    Device state: the current token [B, 1], the write position (int64 [1]), the per-sequence
    visible lengths ``kv_lens`` (int32 [B], = position + 1 during the step) and the output
    token buffer. A replay embeds the token, runs every layer (K/V written at the position,
    attention over the full-capacity cache masked by kv_lens), takes the argmax, stores it,
    and advances the position and lengths, all on the device.
    """

    def __init__(self, model: Decoder, cache: KVCache, max_new_tokens: int):
        if model.attention_name != "student":
            raise ValueError("the graphed decode step runs the student attention kernels")
        self.model, self.cache = model, cache
        dev = model.embedding.device
        b = cache.batch_size
        self.max_new_tokens = max_new_tokens
        self.token = torch.zeros(b, 1, dtype=torch.long, device=dev)
        self.position = torch.zeros(1, dtype=torch.long, device=dev)
        self.kv_lens = torch.zeros(b, dtype=torch.int32, device=dev)
        # Columns past max_new_tokens absorb the capture warm-up's writes.
        self.out = torch.zeros(b, max_new_tokens + self.MAX_WARMUP, dtype=torch.long, device=dev)
        self.out_index = torch.zeros(1, dtype=torch.long, device=dev)
        self.graph = None
        # Host copies of the device position / output column: every step is checked against
        # the cache capacity and the output width on the host before it is launched, so no
        # device-side index ever leaves its tensor.
        self._pos = 0
        self._col = 0

    MAX_WARMUP = 4

    def _advance(self, steps: int):
        if self._pos + steps > self.cache.capacity:
            raise ValueError("KV cache capacity exceeded by the graphed decode steps")
        if self._col + steps > self.out.shape[1]:
            raise ValueError("more graphed decode steps than the output buffer holds")
        self._pos += steps
        self._col += steps

    def _step(self):
        from .operators import student
        model, cache = self.model, self.cache
        cap = cache.capacity
        x = F.embedding(self.token, model.embedding)
        self.kv_lens.copy_((self.position + 1).to(torch.int32).expand_as(self.kv_lens))
        if model.fused_rope:
            tables = (model.rope_cos, model.rope_sin)
            for layer, block in enumerate(model.blocks):
                x = block.forward_fused(x, tables, layer, cache, self.position, self.kv_lens,
                                        fused_qkv=model.fused_qkv)
        else:
            cos, sin = model.rope_tables(self.position)
            for layer, block in enumerate(model.blocks):
                q, k, v = block.project_qkv(x, cos, sin)
                keys, values = cache.append_at(layer, k, v, self.position)
                attended = student.attention(q, keys, values, cap - 1, None, self.kv_lens)
                x = block.finish(x, attended)
        nxt = model.logits(x)[:, -1, :].argmax(dim=-1, keepdim=True)
        self.token.copy_(nxt)
        self.out.index_copy_(1, self.out_index, nxt)
        self.position.add_(1)
        self.out_index.add_(1)

    def prepare(self, first_token: torch.Tensor, out_index: int = 1):
        """Load the state after an eager prefill: the token generated from the prompt, the
        cache length as the next write position, and the output column to write next."""
        self.token.copy_(first_token)
        self.position.fill_(self.cache.length)
        self.out_index.fill_(out_index)
        self.out[:, 0:1].copy_(first_token)
        self._pos, self._col = self.cache.length, out_index

    def capture(self, warmup: int = 2):
        """Capture the step (after `warmup` eager runs on a side stream, which also do the
        one-time device set-up of the kernels). Restores the state the warm-up advanced."""
        if not 0 < warmup <= self.MAX_WARMUP:
            raise ValueError(f"warmup must be in [1, {self.MAX_WARMUP}]")
        saved = (self.token.clone(), self.position.clone(), self.out_index.clone())
        saved_host = (self._pos, self._col)
        self._advance(warmup)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream().wait_stream(side)
        self.token.copy_(saved[0])
        self.position.copy_(saved[1])
        self.out_index.copy_(saved[2])
        self._pos, self._col = saved_host
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        # Capture records the step without running it; the state is unchanged.
        return self

    def replay(self, steps: int):
        if self.graph is None:
            raise RuntimeError("capture() the decode step before replaying it")
        self._advance(steps)
        for _ in range(steps):
            self.graph.replay()

    def tokens(self) -> torch.Tensor:
        """The generated ids so far, [B, columns written]."""
        return self.out[:, :self._col]


# ------------------------------------------------------------------------ generation / timing

def _sync(device):
    if device.type == "cuda":
        torch.cuda.synchronize(device)


@torch.inference_mode()
def generate(model: Decoder, prompt: torch.Tensor, new_tokens: int, graphed: bool = False):
    """Greedy generation (generate.py:9-29 with temperature 0): returns [B, new_tokens] ids."""
    if new_tokens <= 0:
        raise ValueError("new_tokens must be positive")
    cache = model.new_cache(prompt.shape[0], prompt.shape[1] + new_tokens)
    token = model(prompt, cache=cache, last_only=True)[:, -1, :].argmax(dim=-1, keepdim=True)
    if graphed and new_tokens > 1:
        g = GraphedDecode(model, cache, new_tokens)
        g.prepare(token)
        g.capture()
        g.replay(new_tokens - 1)
        return g.tokens().clone()
    out = [token]
    for _ in range(new_tokens - 1):
        token = model(token, cache=cache, last_only=True)[:, -1, :].argmax(dim=-1, keepdim=True)
        out.append(token)
    return torch.cat(out, dim=1)


@torch.inference_mode()
def request(model: Decoder, prompt: torch.Tensor, new_tokens: int, graphed: bool = False):
    """One timed request (benchmarks/model.py:19-37): cache allocation, prefill through the first
    token (TTFT), then the remaining decode steps with no per-token host synchronisation
    (TPOT). Host wall time around device synchronisations. In graphed mode the capture of the
    decode step happens before the timer starts, as a serving loop would hold the graph.

    Entering ``torch.cuda.graph`` empties the caching allocator (``torch.cuda.empty_cache``),
    so the first eager prefill after a capture would allocate every activation buffer through
    cudaMalloc again. One untimed prefill after the capture brings the allocator back to the
    state a serving loop runs in; without it the graphed TTFT measured the re-allocation."""
    device = prompt.device
    g = None
    if graphed:
        # Graphs are bound to cache storage: build the cache and capture before timing.
        cache = model.new_cache(prompt.shape[0], prompt.shape[1] + new_tokens)
        token = model(prompt, cache=cache, last_only=True)[:, -1, :].argmax(dim=-1, keepdim=True)
        g = GraphedDecode(model, cache, new_tokens)
        g.prepare(token)
        g.capture()
        cache.reset()
        model(prompt, cache=cache, last_only=True)
        cache.reset()
    _sync(device)
    start = time.perf_counter()
    if g is None:
        cache = model.new_cache(prompt.shape[0], prompt.shape[1] + new_tokens)
    token = model(prompt, cache=cache, last_only=True)[:, -1, :].argmax(dim=-1, keepdim=True)
    _sync(device)
    first = time.perf_counter()
    if g is None:
        for _ in range(new_tokens - 1):
            token = model(token, cache=cache, last_only=True)[:, -1, :].argmax(dim=-1, keepdim=True)
        tokens = None
    else:
        g.prepare(token)
        g.replay(new_tokens - 1)
        tokens = g.tokens()
    _sync(device)
    end = time.perf_counter()
    b = prompt.shape[0]
    return {"ttft_ms": (first - start) * 1e3,
            "tpot_ms": (end - first) * 1e3 / max(1, new_tokens - 1),
            "request_ms": (end - start) * 1e3,
            "output_tokens_per_second": b * new_tokens / (end - start),
            "decode_tokens_per_second": b * (new_tokens - 1) / (end - first),
            "kv_allocated_bytes": cache.allocated_bytes(),
            "last_tokens": tokens if tokens is not None else token}
