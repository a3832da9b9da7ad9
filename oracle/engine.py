"""ORACLE — test infrastructure only, never part of the product path.

CPU restatement (plain torch on the host) of the reference's paged model step,
used as the timed CPU baseline of the engine workload (``bench.py --workload
engine``) and pinned against the reference's own logits in
``tests/golden/engine_tokens.npz`` (``tests/test_oracle_engine.py``).

It restates, per step and per layer, what src/server/torch_model.py does:
RMSNorm with fp32 statistics cast back (:283-287), bf16-rounded rotary tables
(:199-200, 289-292), Q/K/V projections with bias (:274-276), rotate-half RoPE
(:190-192, 262-264), the per-sequence slot write (PagedKVCache.append :149-153)
and attention (PagedKVCache.attend :155-167 through paged_attention :67-80 for
one token and _read_blocks + attend with _causal_mask :39-64, 295-297 for a
chunk), o_proj, the SwiGLU MLP (:278-281), the final norm and the tied output
projection (:223-229).  ``ReferenceBackend`` restates the reference's paged
backend (src/server/backend/paged.py:21-99) around it over a host pool and the
oracle's allocator, and ``run_for`` the scheduler's admission loop
(src/server/scheduler.py:112-158): no part of the package runs in the baseline.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


class ReferenceModelStep:
    def __init__(self, weights: dict[str, torch.Tensor], dtype: torch.dtype, num_layers: int,
                 num_heads: int, num_kv_heads: int, rope_theta: float, rms_norm_eps: float):
        self.w = {k: v.to(dtype) for k, v in weights.items()}
        self.dtype = dtype
        self.num_layers = num_layers
        self.heads = num_heads
        self.kv_heads = num_kv_heads
        hidden = self.w["model.embed_tokens.weight"].shape[1]
        self.head_dim = hidden // num_heads
        self.eps = rms_norm_eps
        half = torch.arange(0, self.head_dim, 2, dtype=torch.float)
        self.inv_freq = 1.0 / (rope_theta ** (half / self.head_dim))

    # -------------------------------------------------------------- pieces

    def _norm(self, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        f = x.float()
        f = f * torch.rsqrt(f.square().mean(-1, keepdim=True) + self.eps)
        return weight * f.to(x.dtype)

    def _rope_tables(self, positions: torch.Tensor):
        ang = positions[:, None].float() * self.inv_freq
        ang = torch.cat((ang, ang), dim=-1)
        return ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)

    @staticmethod
    def _rotate(x: torch.Tensor) -> torch.Tensor:
        a, b = x.chunk(2, dim=-1)
        return torch.cat((-b, a), dim=-1)

    def _attend_one(self, pool_k, pool_v, table, past, q):
        """q [heads, n, D] at positions past .. past + n - 1 of one sequence."""
        n = q.shape[1]
        total = past + n
        bs = pool_k.shape[2]
        pieces_k, pieces_v = [], []
        for i, block in enumerate(table):
            take = min(bs, total - i * bs)
            if take <= 0:
                break
            pieces_k.append(pool_k[:, block, :take])
            pieces_v.append(pool_v[:, block, :take])
        keys = torch.cat(pieces_k, dim=1).repeat_interleave(self.heads // self.kv_heads, dim=0)
        values = torch.cat(pieces_v, dim=1).repeat_interleave(self.heads // self.kv_heads, dim=0)
        scores = q @ keys.transpose(1, 2) * self.head_dim ** -0.5
        if n > 1:
            future = torch.ones(n, n, dtype=torch.bool).triu(diagonal=1)
            mask = torch.cat((torch.zeros(n, past, dtype=torch.bool), future), dim=1)
            scores = scores.masked_fill(mask, -torch.inf)
        weights = F.softmax(scores, dim=-1, dtype=torch.float32)
        return weights.to(q.dtype) @ values

    # -------------------------------------------------------------- step

    @torch.inference_mode()
    def forward_batch(self, groups) -> torch.Tensor:
        """Last-token logits of each (tokens, cache) group."""
        w = self.w
        for tokens, cache in groups:
            cache.reserve(len(tokens))
        pos = torch.cat([torch.arange(c.length, c.length + len(t)) for t, c in groups])
        cos, sin = self._rope_tables(pos)
        flat = [t for tokens, _ in groups for t in tokens]
        x = w["model.embed_tokens.weight"][flat]
        bounds, start = [], 0
        for tokens, _ in groups:
            bounds.append((start, start + len(tokens)))
            start += len(tokens)
        T, H, Hkv, D = x.shape[0], self.heads, self.kv_heads, self.head_dim
        for layer in range(self.num_layers):
            p = f"model.layers.{layer}."
            h = self._norm(x, w[p + "input_layernorm.weight"])

            def proj(name, heads):
                y = F.linear(h, w[p + f"self_attn.{name}.weight"], w[p + f"self_attn.{name}.bias"])
                return y.view(T, heads, D).transpose(0, 1)

            q, k, v = proj("q_proj", H), proj("k_proj", Hkv), proj("v_proj", Hkv)
            q = q * cos + self._rotate(q) * sin
            k = k * cos + self._rotate(k) * sin
            outs = []
            for (s, e), (_, cache) in zip(bounds, groups):
                pool = cache._pool
                pk, pv = pool.keys[layer], pool.values[layer]
                table = pool.block_table(cache.seq_id)
                for i in range(e - s):
                    block, off = divmod(cache.length + i, pool.block_size)
                    pk[:, table[block], off] = k[:, s + i]
                    pv[:, table[block], off] = v[:, s + i]
                outs.append(self._attend_one(pk, pv, table, cache.length, q[:, s:e]))
            att = torch.cat(outs, dim=1).transpose(0, 1).reshape(T, H * D)
            x = x + F.linear(att, w[p + "self_attn.o_proj.weight"])
            h = self._norm(x, w[p + "post_attention_layernorm.weight"])
            gate = F.silu(F.linear(h, w[p + "mlp.gate_proj.weight"]))
            up = F.linear(h, w[p + "mlp.up_proj.weight"])
            x = x + F.linear(gate * up, w[p + "mlp.down_proj.weight"])
        for tokens, cache in groups:
            cache.advance(len(tokens))
        last = x[[e - 1 for _, e in bounds]]
        return F.linear(self._norm(last, w["model.norm.weight"]), w["model.embed_tokens.weight"])

    def next_tokens(self, groups) -> list[int]:
        return self.forward_batch(groups).float().argmax(dim=-1).tolist()


class _Pool:
    """src/server/torch_model.py:115-137 on the host: [layers, kv_heads, blocks,
    block_size, head_dim] pools and the oracle's restated BlockAllocator."""

    def __init__(self, config, num_blocks: int, block_size: int, dtype: torch.dtype):
        from oracle import Allocator

        shape = (config.num_layers, config.num_kv_heads, num_blocks, block_size, config.head_dim)
        self.keys = torch.zeros(shape, dtype=dtype)
        self.values = torch.zeros(shape, dtype=dtype)
        self.block_size = block_size
        self.allocator = Allocator(num_blocks, block_size)

    @property
    def free_blocks(self) -> int:
        return len(self.allocator.free_list)

    def block_table(self, seq_id: int) -> list[int]:
        return self.allocator.tables[seq_id]

    def new_cache(self, seq_id: int) -> "_Cache":
        return _Cache(self, seq_id)

    def release(self, cache: "_Cache") -> None:
        self.allocator.free(cache.seq_id)


class _Cache:
    """src/server/torch_model.py:140-147, 169-170: length bookkeeping."""

    def __init__(self, pool: _Pool, seq_id: int):
        self._pool = pool
        self.seq_id = seq_id
        self.length = 0

    def reserve(self, count: int) -> None:
        self._pool.allocator.allocate(self.seq_id, self.length + count)

    def advance(self, count: int) -> None:
        self.length += count


class ReferenceBackend:
    """src/server/backend/paged.py:21-99 restated over ``ReferenceModelStep``:
    generating sequences' next tokens first, then prompt pieces under the
    prefill budget in sequence order; a sequence whose prompt is used up gets
    its greedy token; release frees its blocks.  Token ids only (end of
    generation: Qwen2.5's 151643 / 151645)."""

    END_OF_GENERATION = frozenset({151643, 151645})

    def __init__(self, model: ReferenceModelStep, pool: _Pool, prefill_chunk: int):
        self._model = model
        self.pool = pool
        self._prefill_chunk = prefill_chunk
        self._next_id = 0
        self._sequences: dict[int, dict] = {}

    def start_sequence(self, prompt_tokens: list[int]) -> int:
        seq_id, self._next_id = self._next_id, self._next_id + 1
        cache = self.pool.new_cache(seq_id)
        cache.reserve(0)
        self._sequences[seq_id] = dict(cache=cache, pending=list(prompt_tokens), next=None,
                                       finished=False)
        return seq_id

    def step(self) -> dict[int, tuple[int, bool]]:
        batch = [(s, [q["next"]]) for s, q in self._sequences.items()
                 if not q["pending"] and not q["finished"]]
        budget = self._prefill_chunk
        for s, q in self._sequences.items():
            take = min(budget, len(q["pending"]))
            if take:
                batch.append((s, q["pending"][:take]))
                del q["pending"][:take]
                budget -= take
        if not batch:
            return {}
        tokens = self._model.next_tokens([(t, self._sequences[s]["cache"]) for s, t in batch])
        outputs = {}
        for (s, _), token in zip(batch, tokens):
            q = self._sequences[s]
            if not q["pending"]:
                q["next"] = token
                q["finished"] = token in self.END_OF_GENERATION
                outputs[s] = (token, q["finished"])
        return outputs

    def release_sequence(self, seq_id: int) -> None:
        self.pool.release(self._sequences.pop(seq_id)["cache"])


def cpu_backend(weights, dtype, config, num_blocks: int, block_size: int, prefill_chunk: int):
    """The restated reference backend over ``ReferenceModelStep`` with a host
    pool of `dtype` (the reference's own pool is bf16; fp32 serves parity)."""
    model = ReferenceModelStep(weights, dtype, config.num_layers, config.num_heads,
                               config.num_kv_heads, config.rope_theta, config.rms_norm_eps)
    return ReferenceBackend(model, _Pool(config, num_blocks, block_size, dtype), prefill_chunk)


def run_for(backend: ReferenceBackend, specs, max_concurrent: int, num_blocks: int,
            block_size: int, seconds: float, warmup: bool = True) -> tuple[int, int, float]:
    """src/server/scheduler.py:112-158 (BatchingScheduler, its BlockBudget
    src/server/kv_budget.py) restated as a plain loop over queued requests:
    admit from the head while under max_concurrent and the budget reserves
    ceil((prompt + max_tokens) / block_size) blocks, step, count tokens,
    complete at max_tokens or end of generation.  Steps until `seconds` pass
    or every request is done; returns (tokens generated, steps, elapsed
    seconds), the first step untimed when `warmup`."""
    import time
    from collections import deque

    waiting = deque((list(p), int(m)) for p, m in specs)
    active: dict[int, list] = {}
    available = num_blocks
    blocks = lambda p, m: -(-(len(p) + m) // block_size)  # noqa: E731

    def turn() -> int:
        nonlocal available
        while (waiting and len(active) < max_concurrent
               and blocks(*waiting[0]) <= available):
            p, m = waiting.popleft()
            available -= blocks(p, m)
            active[backend.start_sequence(p)] = [p, m, 0]
        outputs = backend.step()
        for s, (_, finished) in outputs.items():
            req = active[s]
            req[2] += 1
            if finished or req[2] >= req[1]:
                available += blocks(req[0], req[1])
                del active[s]
                backend.release_sequence(s)
        return len(outputs)

    if warmup:
        turn()
    generated, steps = 0, 0
    start = time.perf_counter()
    while (waiting or active) and time.perf_counter() - start < seconds:
        generated += turn()
        steps += 1
    return generated, steps, time.perf_counter() - start
