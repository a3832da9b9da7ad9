"""The paged-backend model step on the GPU: the reference's TorchModel with its
per-sequence attention loop replaced by one batched call per layer.

Mirrors src/server/torch_model.py: ``ModelConfig`` (:13-36), ``PagedKVPool`` /
``PagedKVCache`` (:115-170) and ``TorchModel`` (:195-297), with the same layer
maths and rounding points (bf16 rotary tables, fp32 RMSNorm statistics cast back
to the hidden dtype, SwiGLU MLP, tied output embedding).  What changes is where
the work runs and how a step is assembled (``_hidden_states`` :231-247):

* block tables and context lengths live on the device
  (``BlockAllocator(device=...)``), and one ``step_metadata`` launch derives the
  ragged-batch metadata (chunk offsets, positions, slot mapping, context
  lengths) that the reference rebuilt in Python every step;
* each layer rotates q and k and writes the step's K/V rows in one
  ``rope_append`` launch (torch_model.py:262-264, PagedKVCache.append
  :149-153) and attends with one batched decode launch for the single-token
  rows plus one chunked-prefill launch for the prompt chunks
  (PagedKVCache.attend, :155-167), instead of 2 x B Python-level calls;
* the residual adds, RMSNorms (:283-287), embedding gather and SwiGLU gating
  run in fused kernels with the reference's rounding points, so a layer is
  five of this package's launches around four library GEMMs;
* the last-token logits are reduced to greedy token ids on the device
  (PagedBackend._next_output, backend/paged.py:95-99), so only B ints cross
  PCIe per step.

The projections and the MLP are plain library GEMMs (cuBLAS through torch);
everything else in a step is this package's kernels.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import torch
import torch.nn.functional as F

from . import ops
from .block_allocator import BlockAllocator


@dataclass(frozen=True)
class ModelConfig:
    """src/server/torch_model.py:13-36 (the same fields and head_dim rule)."""

    num_layers: int
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    rope_theta: float
    rms_norm_eps: float

    @classmethod
    def from_file(cls, path: Path) -> "ModelConfig":
        config = json.loads(Path(path).read_text())
        return cls(
            num_layers=config["num_hidden_layers"],
            hidden_size=config["hidden_size"],
            num_heads=config["num_attention_heads"],
            num_kv_heads=config["num_key_value_heads"],
            rope_theta=config["rope_theta"],
            rms_norm_eps=config["rms_norm_eps"],
        )

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


# The Qwen2.5-0.5B shape (24 layers, hidden 896, 14 / 2 heads, head_dim 64).
QWEN25_05B = ModelConfig(num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
QWEN25_05B_VOCAB = 151936
QWEN25_05B_INTERMEDIATE = 4864


def weight_names(config: ModelConfig) -> list[str]:
    """Parameter names in checkpoint order (the reference's key names)."""
    names = ["model.embed_tokens.weight"]
    for layer in range(config.num_layers):
        p = f"model.layers.{layer}."
        names += [p + "input_layernorm.weight"]
        for proj in ("q_proj", "k_proj", "v_proj"):
            names += [p + f"self_attn.{proj}.weight", p + f"self_attn.{proj}.bias"]
        names += [p + "self_attn.o_proj.weight", p + "post_attention_layernorm.weight",
                  p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", p + "mlp.down_proj.weight"]
    names.append("model.norm.weight")
    return names


def weight_shapes(config: ModelConfig, vocab_size: int, intermediate_size: int) -> dict[str, tuple]:
    hidden, kv = config.hidden_size, config.num_kv_heads * config.head_dim
    shapes = {"model.embed_tokens.weight": (vocab_size, hidden), "model.norm.weight": (hidden,)}
    for layer in range(config.num_layers):
        p = f"model.layers.{layer}."
        shapes.update({
            p + "input_layernorm.weight": (hidden,),
            p + "post_attention_layernorm.weight": (hidden,),
            p + "self_attn.q_proj.weight": (hidden, hidden), p + "self_attn.q_proj.bias": (hidden,),
            p + "self_attn.k_proj.weight": (kv, hidden), p + "self_attn.k_proj.bias": (kv,),
            p + "self_attn.v_proj.weight": (kv, hidden), p + "self_attn.v_proj.bias": (kv,),
            p + "self_attn.o_proj.weight": (hidden, hidden),
            p + "mlp.gate_proj.weight": (intermediate_size, hidden),
            p + "mlp.up_proj.weight": (intermediate_size, hidden),
            p + "mlp.down_proj.weight": (hidden, intermediate_size),
        })
    return shapes


def random_weights(config: ModelConfig = QWEN25_05B, vocab_size: int = QWEN25_05B_VOCAB,
                   intermediate_size: int = QWEN25_05B_INTERMEDIATE, seed: int = 0,
                   std: float = 0.02) -> dict[str, torch.Tensor]:
    """Random-init fp32 CPU weights: every matrix, the embedding and every bias
    N(0, std) drawn from one ``torch.Generator`` seeded ``seed`` in checkpoint
    order (``weight_names``); RMSNorm weights are 1."""
    g = torch.Generator().manual_seed(seed)
    shapes = weight_shapes(config, vocab_size, intermediate_size)
    weights = {}
    for name in weight_names(config):
        if name.endswith("norm.weight"):
            weights[name] = torch.ones(shapes[name])
        else:
            weights[name] = torch.randn(shapes[name], generator=g) * std
    return weights


def load_safetensors(path: Path) -> dict[str, torch.Tensor]:
    """BF16 safetensors reader (the checkpoint format the reference loads,
    src/server/torch_model.py:173-187)."""
    data = bytearray(Path(path).read_bytes())
    header_size = struct.unpack_from("<Q", data)[0]
    header = json.loads(data[8: 8 + header_size])
    header.pop("__metadata__", None)
    weights = {}
    for name, entry in header.items():
        if entry["dtype"] != "BF16":
            raise ValueError(f"{name} has unsupported dtype {entry['dtype']}")
        start, end = entry["data_offsets"]
        tensor = torch.frombuffer(data, dtype=torch.bfloat16, count=(end - start) // 2,
                                  offset=8 + header_size + start)
        weights[name] = tensor.reshape(entry["shape"])
    return weights


class PagedKVPool:
    """Device-resident K/V pool [layers, kv_heads, blocks, block_size, head_dim]
    with the reference's allocator and a device mirror of its block tables
    (src/server/torch_model.py:115-137).  ``dtype`` is bf16 as in the reference;
    fp32 pools serve fp32 parity runs."""

    def __init__(self, config: ModelConfig, num_blocks: int, block_size: int,
                 device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16,
                 max_seqs: int = 256, max_blocks_per_seq: int | None = None):
        self.device = torch.device(device)
        shape = (config.num_layers, config.num_kv_heads, num_blocks, block_size, config.head_dim)
        self.keys = torch.zeros(shape, dtype=dtype, device=self.device)
        self.values = torch.zeros(shape, dtype=dtype, device=self.device)
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.allocator = BlockAllocator(num_blocks, block_size, max_seqs=max_seqs,
                                        max_blocks_per_seq=max_blocks_per_seq or num_blocks,
                                        device=self.device)
        # Greedy token ids of the last step run on this pool, in that step's row
        # layout: a step may take a row's input token from here (a token
        # reference) before the host has read it.  Rows: every live sequence,
        # plus the padding of a graph-captured step.
        self.last_ids = torch.zeros(max_seqs + 64, dtype=torch.int32, device=self.device)

    @property
    def free_blocks(self) -> int:
        return self.allocator.free_blocks

    def block_table(self, seq_id: int) -> list[int]:
        return self.allocator.block_table(seq_id)

    def new_cache(self, seq_id: int) -> "PagedKVCache":
        return PagedKVCache(self, seq_id)

    def release(self, cache: "PagedKVCache") -> None:
        self.allocator.free(cache.seq_id)


class PagedKVCache:
    """One sequence's view of the pool (src/server/torch_model.py:140-170).  The
    K/V writes and attention of a step are batched by ``TorchModel``; the cache
    keeps the length bookkeeping."""

    def __init__(self, pool: PagedKVPool, seq_id: int):
        self._pool = pool
        self.seq_id = seq_id
        self.length = 0

    def reserve(self, count: int) -> None:
        self._pool.allocator.allocate(self.seq_id, self.length + count)

    def advance(self, count: int) -> None:
        self.length += count


class PendingTokens:
    """The greedy token ids of a launched step: ``result()`` waits for the step
    and returns one id per group; ``ref(i)`` is the token reference (a negative
    input token) through which the next step can take group i's id on the
    device before the host has it."""

    def __init__(self, model: "TorchModel", host: torch.Tensor, status: torch.Tensor, event,
                 index: list[int]):
        self._model = model
        self._host = host
        self._status = status  # the status words of the step's workspaces, copied after it
        self._event = event
        self._index = index
        self._values = None

    def ref(self, i: int) -> int:
        return -1 - self._index[i]

    def result(self) -> list[int]:
        if self._values is None:
            self._event.synchronize()
            if bool(self._status.any()):
                self._model._raise_status()
            vals = self._host.tolist()
            self._values = [vals[j] for j in self._index]
        return self._values


class TorchModel:
    """The reference TorchModel (src/server/torch_model.py:195-297) on one GPU,
    over a ``PagedKVPool`` on the same device.  ``dtype`` is the compute dtype
    of the hidden states and weights (bf16 as the checkpoint, or fp32)."""

    def __init__(self, config: ModelConfig, weights: dict[str, torch.Tensor],
                 device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16,
                 max_position: int = 32768, step_graphs: bool = True,
                 max_graph_batch: int = 256, max_graph_prefill: int = 512,
                 max_graph_chunks: int = 8):
        self.config = config
        self.device = torch.device(device)
        self.dtype = dtype
        w = {k: v.to(device=self.device, dtype=dtype) for k, v in weights.items()}
        self.embed = w["model.embed_tokens.weight"]
        self.final_norm = w["model.norm.weight"]
        self.layers = []
        for layer in range(config.num_layers):
            p = f"model.layers.{layer}."
            a = p + "self_attn."
            self.layers.append(dict(
                ln1=w[p + "input_layernorm.weight"],
                ln2=w[p + "post_attention_layernorm.weight"],
                # Q, K and V share one GEMM; gate and up share another.
                qkv_w=torch.cat([w[a + "q_proj.weight"], w[a + "k_proj.weight"],
                                 w[a + "v_proj.weight"]]).contiguous(),
                qkv_b=torch.cat([w[a + "q_proj.bias"], w[a + "k_proj.bias"],
                                 w[a + "v_proj.bias"]]).contiguous(),
                o_w=w[a + "o_proj.weight"],
                gate_up_w=torch.cat([w[p + "mlp.gate_proj.weight"],
                                     w[p + "mlp.up_proj.weight"]]).contiguous(),
                down_w=w[p + "mlp.down_proj.weight"],
            ))
        self.intermediate_size = self.layers[0]["down_w"].shape[1] if self.layers else 0
        self.vocab_size = self.embed.shape[0]
        # Rotary tables exactly as the reference makes them (fp32 angles on the
        # CPU, cos/sin rounded to bf16, torch_model.py:199-200, 289-292), built
        # once for every position and gathered per step on the device.
        steps = torch.arange(0, config.head_dim, 2, dtype=torch.float)
        inverse_frequencies = 1.0 / (config.rope_theta ** (steps / config.head_dim))
        positions = torch.arange(max_position)
        frequencies = positions[:, None].float() * inverse_frequencies
        angles = torch.cat((frequencies, frequencies), dim=-1)
        self.cos = angles.cos().to(torch.bfloat16).to(device=self.device, dtype=dtype)
        self.sin = angles.sin().to(torch.bfloat16).to(device=self.device, dtype=dtype)
        self.max_position = max_position
        # Per-step accounting for benchmarks: forwards, tokens and rows
        # processed, attention FLOPs (QK^T + PV over visible keys), launches of
        # this package's kernels, bytes copied host->device and device->host.
        self.stats = dict(steps=0, tokens=0, rows=0, attn_flops=0, launches=0, h2d_bytes=0,
                          d2h_bytes=0)
        self._host = None  # pinned staging buffer for per-step row metadata
        self._host_free = None  # event: the last copy out of it has completed
        # Steps replay CUDA graphs captured per padded shape (decode rows, prompt
        # chunks, prompt tokens), on a stream no eager call uses; steps beyond
        # max_graph_batch decode rows, max_graph_chunks chunks or
        # max_graph_prefill prompt tokens run eagerly.
        self.step_graphs = step_graphs and self.device.type == "cuda"
        self.max_graph_batch = max_graph_batch
        self.max_graph_prefill = max_graph_prefill
        self.max_graph_chunks = max_graph_chunks
        self._graphs: dict[tuple, tuple] = {}
        self._graph_stream = None
        self._graph_pool = None
        self._graph_ws = None
        self._hosts = None  # pinned buffers for pending token ids
        self._host_turn = 0

    @classmethod
    def load(cls, model_dir: Path, device="cuda", dtype=torch.bfloat16) -> "TorchModel":
        model_dir = Path(model_dir)
        config = ModelConfig.from_file(model_dir / "config.json")
        return cls(config, load_safetensors(model_dir / "model.safetensors"), device, dtype)

    # ---------------------------------------------------------------- public

    @torch.inference_mode()
    def forward_batch(self, groups: list[tuple[list[int], PagedKVCache]]) -> torch.Tensor:
        """Each (tokens, cache) pair's last-token logits [B, vocab] on the device
        (torch_model.py:223-229)."""
        last = self._last_hidden(groups)
        return F.linear(last, self.embed)

    @torch.inference_mode()
    def next_tokens(self, groups: list[tuple[list[int], PagedKVCache]]) -> list[int]:
        """Greedy next token of each group: argmax of the last-token logits
        (first index on ties; bf16 -> fp32 is exact, so the argmax of the
        model-dtype logits is the reference's argmax of logits.float()),
        reduced on the device.  Steps within the graph limits replay a
        captured step graph."""
        return self.launch_tokens(groups).result()

    @torch.inference_mode()
    def launch_tokens(self, groups: list[tuple[list[int], PagedKVCache]]) -> PendingTokens:
        """``next_tokens`` without waiting: launches the step and returns its
        pending ids.  An input token t < 0 of a group is a token reference: the
        id of row -1 - t of the last step launched on this pool (see
        ``PendingTokens.ref``)."""
        key = self._graph_key([len(tokens) for tokens, _ in groups]) if self.step_graphs else None
        if key is not None:
            return self._graph_step(groups, key)
        pool = groups[0][1]._pool
        logits = self.forward_batch(groups)
        ids = ops.argmax_rows(logits)
        pool.last_ids[: ids.numel()].copy_(ids)
        return self._pending(ids, list(range(len(groups))))

    def _pending(self, ids: torch.Tensor, index: list[int]) -> PendingTokens:
        """Copies `ids` to one of a few pinned buffers and records the event the
        host waits on; at most len(self._hosts) - 1 steps may be pending."""
        n = ids.numel()
        if self._hosts is None or self._hosts[0].numel() < n + 2:
            self._hosts = [torch.empty(max(n + 2, 1024), dtype=torch.int32, pin_memory=True)
                           for _ in range(3)]
        buf = self._hosts[self._host_turn]
        self._host_turn = (self._host_turn + 1) % len(self._hosts)
        host, status = buf[:n], buf[n: n + 2]
        host.copy_(ids, non_blocking=True)
        # Kernels report bad input in the status word of their stream's
        # workspace (eager calls: this stream; graph replays: the capture
        # stream's): copied after the step, read with the ids.
        status[0].copy_(ops.workspace_for(self.device, 0)[:4].view(torch.int32)[0],
                        non_blocking=True)
        if self._graph_ws is not None:
            status[1].copy_(self._graph_ws[:4].view(torch.int32)[0], non_blocking=True)
        else:
            status[1].fill_(0)
        self.stats["d2h_bytes"] += 4 * n
        event = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self.device))
        return PendingTokens(self, host, status, event, index)

    def _raise_status(self) -> None:
        """Takes (and clears) both status words, raising for the set bits."""
        ops.take_status(self.device)
        if self._graph_stream is not None:
            with torch.cuda.stream(self._graph_stream):
                ops.take_status(self.device)

    # ---------------------------------------------------------------- step

    def _stage(self, values: list[int]) -> torch.Tensor:
        """One pinned host buffer -> one H2D copy of the step's int32 metadata."""
        n = len(values)
        if self._host_free is not None:
            self._host_free.synchronize()  # the previous step's copy has left the buffer
        if self._host is None or self._host.numel() < n:
            self._host = torch.empty(max(n, 1024) * 2, dtype=torch.int32, pin_memory=True)
        self._host[:n] = torch.tensor(values, dtype=torch.int32)
        staged = self._host[:n].to(self.device, non_blocking=True)
        self.stats["h2d_bytes"] += 4 * n
        self._host_free = torch.cuda.Event()
        self._host_free.record(torch.cuda.current_stream(self.device))
        return staged

    def _last_hidden(self, groups) -> torch.Tensor:
        config = self.config
        pool = groups[0][1]._pool
        for tokens, cache in groups:
            cache.reserve(len(tokens))
        alloc = pool.allocator
        self.stats["h2d_bytes"] += 16 * alloc.sync_device()
        launches = ops.kernel_launches()
        R = len(groups)
        lengths = [len(tokens) for tokens, _ in groups]
        T = sum(lengths)
        starts = [cache.length for _, cache in groups]
        if max(s + n for s, n in zip(starts, lengths)) > self.max_position:
            raise RuntimeError(f"positions beyond the rotary table ({self.max_position})")
        rows = [alloc.row(cache.seq_id) for _, cache in groups]
        flat = [t for tokens, _ in groups for t in tokens]
        ends = [sum(lengths[: i + 1]) - 1 for i in range(R)]
        # Context lengths after the step are known here: the decode kernel gets
        # them as final at launch (lens_ready) and partitions its work while the
        # K/V write before it is still running.
        after = [st + n for st, n in zip(starts, lengths)]
        staged = self._stage(rows + starts + lengths + ends + after + flat)
        rows_d, start_d, n_d, ends_d, ctx_d, tokens_d = (
            staged[:R], staged[R:2 * R], staged[2 * R:3 * R], staged[3 * R:4 * R],
            staged[4 * R:5 * R], staged[5 * R:])
        # Leading single-token rows run through the batched decode kernel, the
        # rest (prompt chunks) through the chunked-prefill kernel.
        n_dec = 0
        while n_dec < R and lengths[n_dec] == 1:
            n_dec += 1
        if n_dec == R:
            # One token per row: positions are the start positions; one locate
            # launch gives the slots.
            positions = start_d
            _, slots = ops.decode_append(None, None, pool.keys[0], pool.values[0],
                                         alloc.device_tables, start_d, seq_rows=rows_d)
            cu_q = ctx = None
        else:
            cu_q, positions, slots, ctx = ops.step_metadata(
                alloc.device_tables, start_d, n_d, T, pool.block_size, pool.num_blocks,
                seq_rows=rows_d)
        max_chunk = max(lengths[n_dec:], default=0)
        pre_cu = (cu_q[n_dec:] - n_dec) if n_dec < R else None

        def attend(q, kp, vp, attended):
            if n_dec:
                ops.paged_attention_batched(q[:n_dec], kp, vp, alloc.device_tables, ctx_d[:n_dec],
                                            config.head_dim ** -0.5, seq_rows=rows_d[:n_dec],
                                            out=attended[:n_dec], lens_ready=True,
                                            after_append=True)
            if n_dec < R:
                ops.prefill_attention(q[n_dec:], kp, vp, alloc.device_tables, pre_cu,
                                      ctx[n_dec:], config.head_dim ** -0.5,
                                      max_query_len=max_chunk, seq_rows=rows_d[n_dec:],
                                      out=attended[n_dec:])

        last = self._layers(pool, self._resolve(pool, tokens_d), positions, slots, ends_d, attend)
        for (tokens, cache) in groups:
            cache.advance(len(tokens))
        st = self.stats
        st["steps"] += 1
        st["tokens"] += T
        st["rows"] += R
        st["attn_flops"] += config.num_layers * 4 * config.num_heads * config.head_dim * sum(
            n * s + n * (n + 1) // 2 for s, n in zip(starts, lengths))
        st["launches"] += ops.kernel_launches() - launches
        return last

    @staticmethod
    def _resolve(pool: PagedKVPool, tokens: torch.Tensor) -> torch.Tensor:
        """Token references (t < 0: row -1 - t of the pool's last ids) replaced by
        their ids, on the device."""
        src = (-1 - tokens).clamp_(min=0).long()
        return torch.where(tokens < 0, pool.last_ids.index_select(0, src), tokens)

    def _layers(self, pool: PagedKVPool, tokens, positions, slots, last_rows, attend):
        """The decoder stack over T tokens (torch_model.py:233-248, 250-287) with
        the residual adds, RMSNorms, rotary embedding, K/V append and SwiGLU
        gating in this package's fused kernels and the projections in library
        GEMMs.  ``attend(q, key_pool, value_pool, out)`` runs one layer's paged
        attention.  Returns the final-normed hidden states of rows last_rows."""
        config = self.config
        H, D, eps = config.num_heads, config.head_dim, config.rms_norm_eps
        T = tokens.numel()
        # Residual stream; layer 0's norm also gathers the embedding rows into it.
        hidden = torch.empty((T, config.hidden_size), dtype=self.dtype, device=self.device)
        attended = torch.empty((T, H, D), dtype=self.dtype, device=self.device)
        q = torch.empty((T, H, D), dtype=self.dtype, device=self.device)
        delta = None  # the previous sublayer's output, added before the next norm
        for layer, lw in enumerate(self.layers):
            if layer == 0:
                normed = ops.rms_norm(self.embed, lw["ln1"], eps, row_index=tokens, sum_out=hidden)
            else:
                normed = ops.rms_norm(hidden, lw["ln1"], eps, add=delta, sum_out=hidden)
            qkv = F.linear(normed, lw["qkv_w"], lw["qkv_b"])
            kp, vp = pool.keys[layer], pool.values[layer]
            ops.rope_append(qkv, self.cos, self.sin, positions, slots, kp, vp, H, query_out=q)
            attend(q, kp, vp, attended)
            delta = F.linear(attended.view(T, H * D), lw["o_w"])
            normed = ops.rms_norm(hidden, lw["ln2"], eps, add=delta, sum_out=hidden)
            delta = F.linear(ops.silu_mul(F.linear(normed, lw["gate_up_w"])), lw["down_w"])
        return ops.rms_norm(hidden, self.final_norm, eps, add=delta, row_index=last_rows)

    # ---------------------------------------------------------------- step graphs

    def _decode_bucket(self, n: int) -> int:
        """Padded decode rows: powers of two to 32, then multiples of 32."""
        if n == 0:
            return 0
        b = 1
        while b < min(n, 32):
            b *= 2
        if n > 32:
            b = -(-n // 32) * 32
        return min(b, self.max_graph_batch)

    def _graph_key(self, lengths: list[int]):
        """(decode rows, chunk rows, chunk tokens) of the graph that serves a
        step with these per-row token counts, or None (run eagerly)."""
        n_dec = 0
        while n_dec < len(lengths) and lengths[n_dec] == 1:
            n_dec += 1
        if n_dec > self.max_graph_batch:
            return None
        chunks = lengths[n_dec:]
        if not chunks:
            return (self._decode_bucket(n_dec), 0, 0)
        tok = sum(chunks)
        if len(chunks) > self.max_graph_chunks or tok > self.max_graph_prefill:
            return None
        rows = 1
        while rows < len(chunks):
            rows *= 2
        q = 64
        while q < tok:
            q *= 2
        return (self._decode_bucket(n_dec), rows, q)

    def _graph_forward(self, pool: PagedKVPool, key, inputs: torch.Tensor) -> torch.Tensor:
        """Greedy ids (int32 [B + P], on the device) of one padded step: B
        decode rows then P prompt-chunk rows holding up to Q tokens, described
        by the int32 ``inputs`` (see ``_graph_inputs``).  Launches only (no host
        synchronisation), so it can be captured."""
        config = self.config
        B, P, Q = key
        R, T = B + P, B + Q
        alloc = pool.allocator
        rows, start, n_new, after, ends, tokens = inputs.split([R, R, R, B, R, T])
        cu_q, positions, slots, ctx = ops.step_metadata(
            alloc.device_tables, start, n_new, T, pool.block_size, pool.num_blocks,
            seq_rows=rows)
        pre_cu = cu_q[B:] - B if P else None
        scale = config.head_dim ** -0.5

        def attend(q, kp, vp, attended):
            if B:
                ops.paged_attention_batched(q[:B], kp, vp, alloc.device_tables, after, scale,
                                            seq_rows=rows[:B], out=attended[:B], lens_ready=True,
                                            after_append=True)
            if P:
                ops.prefill_attention(q[B:], kp, vp, alloc.device_tables, pre_cu, ctx[B:], scale,
                                      max_query_len=Q, seq_rows=rows[B:], out=attended[B:])

        last = self._layers(pool, self._resolve(pool, tokens), positions, slots, ends, attend)
        ids = ops.argmax_rows(F.linear(last, self.embed))
        pool.last_ids[:R].copy_(ids)
        return ids

    @staticmethod
    def _graph_inputs(key, rows, starts, lengths, n_dec, tokens) -> list[int]:
        """The int32 input vector of a padded step: rows | start | n_new (R
        each) | context after the step of the decode rows (B) | token index of
        each row's last token (R) | tokens (T).  Padding rows have start -1
        (they read and write nothing); padding tokens are 0."""
        B, P, Q = key
        pd, pp = B - n_dec, P - (len(rows) - n_dec)
        lengths_p = lengths[n_dec:]
        ends, acc = list(range(n_dec)) + [0] * pd, B
        for n in lengths_p:
            acc += n
            ends.append(acc - 1)
        flat_p = [t for ts in tokens[n_dec:] for t in ts]
        return (rows[:n_dec] + [0] * pd + rows[n_dec:] + [0] * pp
                + starts[:n_dec] + [-1] * pd + starts[n_dec:] + [-1] * pp
                + [1] * B + lengths_p + [0] * pp
                + [s + 1 for s in starts[:n_dec]] + [0] * pd
                + ends + [0] * pp
                + [ts[0] for ts in tokens[:n_dec]] + [0] * pd + flat_p + [0] * (Q - len(flat_p)))

    def _reserve_graph_workspace(self, block_size: int) -> None:
        """Sizes the graph stream's workspace for every graph shape before the
        first capture: a captured launch keeps the buffer's address.  (A small
        batch of chunks may need more than a large one: its key ranges split.)"""
        c = self.config
        need = ops.decode_workspace_bytes(self.max_graph_batch, c.num_heads, c.num_kv_heads,
                                          c.head_dim, block_size, self.dtype)
        for rows in _powers_of_two(1, self.max_graph_chunks):
            for q in _powers_of_two(64, self.max_graph_prefill):
                need = max(need, ops.prefill_workspace_bytes(
                    q, rows, q, c.num_heads, c.num_kv_heads, c.head_dim, block_size, self.dtype))
        self._graph_ws = ops.workspace_for(self.device, need)

    @torch.inference_mode()
    def warm_graphs(self, pool: PagedKVPool) -> int:
        """Captures the step graph of every padded shape for `pool` now, so no
        later step waits for a capture; returns how many there are."""
        if not self.step_graphs:
            return 0
        decode = sorted({self._decode_bucket(n) for n in range(self.max_graph_batch + 1)})
        keys = [(b, 0, 0) for b in decode if b] + [
            (b, rows, q) for b in decode for rows in _powers_of_two(1, self.max_graph_chunks)
            for q in _powers_of_two(64, self.max_graph_prefill)]
        for key in keys:
            if (id(pool),) + key not in self._graphs:
                self._capture(pool, key)
        return len(keys)

    def _capture(self, pool: PagedKVPool, key):
        if self._graph_stream is None:
            self._graph_stream = torch.cuda.Stream(self.device)
            self._graph_pool = torch.cuda.graph_pool_handle()
        stream = self._graph_stream
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            if self._graph_ws is None:
                self._reserve_graph_workspace(pool.block_size)
            B, P, Q = key
            R = B + P
            # An all-padding step while warming up and capturing: nothing is
            # read from or written to the pool.
            inputs = torch.tensor([0] * R + [-1] * R + [1] * B + [0] * P + [0] * B + [0] * R
                                  + [0] * (B + Q), dtype=torch.int32, device=self.device)
            # The warm-up run writes its (padding) ids over the pool's last ids,
            # which the step about to replay may still read by reference.
            saved = pool.last_ids.clone()
            self._graph_forward(pool, key, inputs)
            pool.last_ids.copy_(saved)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            before = ops.kernel_launches()
            with torch.cuda.graph(graph, pool=self._graph_pool, stream=stream):
                ids = self._graph_forward(pool, key, inputs)
            launches = ops.kernel_launches() - before
            if ops.workspace_for(self.device, 0).data_ptr() != self._graph_ws.data_ptr():
                raise RuntimeError("the graph workspace moved during capture")
            ops.take_status(self.device)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        entry = (inputs, graph, ids, launches)
        self._graphs[(id(pool),) + key] = entry
        return entry

    def _graph_step(self, groups, key) -> PendingTokens:
        config = self.config
        pool = groups[0][1]._pool
        entry = self._graphs.get((id(pool),) + key)
        if entry is None:
            entry = self._capture(pool, key)
        inputs, graph, ids, graph_launches = entry
        for tokens, cache in groups:
            cache.reserve(len(tokens))
        alloc = pool.allocator
        self.stats["h2d_bytes"] += 16 * alloc.sync_device()
        lengths = [len(tokens) for tokens, _ in groups]
        starts = [cache.length for _, cache in groups]
        if max(s + n for s, n in zip(starts, lengths)) > self.max_position:
            raise RuntimeError(f"positions beyond the rotary table ({self.max_position})")
        n_dec = 0
        while n_dec < len(lengths) and lengths[n_dec] == 1:
            n_dec += 1
        rows = [alloc.row(cache.seq_id) for _, cache in groups]
        values = self._graph_inputs(key, rows, starts, lengths, n_dec,
                                    [tokens for tokens, _ in groups])
        inputs.copy_(self._stage(values))
        graph.replay()
        B = key[0]
        for tokens, cache in groups:
            cache.advance(len(tokens))
        st = self.stats
        st["steps"] += 1
        st["tokens"] += sum(lengths)
        st["rows"] += len(groups)
        st["attn_flops"] += config.num_layers * 4 * config.num_heads * config.head_dim * sum(
            n * s + n * (n + 1) // 2 for s, n in zip(starts, lengths))
        st["launches"] += graph_launches
        index = list(range(n_dec)) + list(range(B, B + len(groups) - n_dec))
        return self._pending(ids, index)


def _powers_of_two(lo: int, limit: int) -> list[int]:
    """lo, 2 lo, ... up to the first value >= limit (the graph buckets)."""
    out = [lo]
    while out[-1] < limit:
        out.append(out[-1] * 2)
    return out


__all__ = ["ModelConfig", "PagedKVPool", "PagedKVCache", "TorchModel", "QWEN25_05B",
           "random_weights", "weight_names", "load_safetensors"]
