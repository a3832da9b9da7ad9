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
projection (:223-229).  The pool and the block tables are the ones of the
``PagedKVCache`` objects it is given (the package's bookkeeping, kept on CPU).
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
        # Interface the package's PagedBackend expects of a model.
        self.device = torch.device("cpu")
        self.max_position = 1 << 20

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

    def launch_tokens(self, groups) -> "_Done":
        """The backend's launch interface, computed at once (the CPU backend
        runs the plain loop: every input token is an id, never a reference)."""
        if any(t < 0 for tokens, _ in groups for t in tokens):
            raise ValueError("the reference model step takes token ids only")
        return _Done(self.next_tokens(groups))


class _Done:
    def __init__(self, values: list[int]):
        self._values = values

    def ref(self, i: int) -> int:
        return -1 - i

    def result(self) -> list[int]:
        return self._values


def cpu_backend(weights, dtype, config, num_blocks: int, block_size: int, prefill_chunk: int,
                max_seqs: int = 256):
    """The package's PagedBackend bookkeeping (reference batch composition and
    allocator) over ``ReferenceModelStep`` with a CPU pool."""
    from batchstream_inference_engine_b200.backend import PagedBackend

    model = ReferenceModelStep(weights, dtype, config.num_layers, config.num_heads,
                               config.num_kv_heads, config.rope_theta, config.rms_norm_eps)
    model.config = config
    model.dtype = dtype
    return PagedBackend(model, num_blocks, block_size, prefill_chunk, max_seqs=max_seqs)
