"""``PagedBackend`` on the GPU: the reference's paged backend
(src/server/backend/paged.py:21-99) over this package's ``TorchModel``.

Same batch composition (every generating sequence's next token first, then
prompt chunks under the ``prefill_chunk`` token budget, in sequence order),
same outputs (one ``StepOutput`` per sequence whose prompt is fully consumed),
same release rules.  The greedy argmax runs on the device and the step returns
after one copy of B token ids.

Tokenization is not on the attention path: the reference takes it from a GGUF
vocabulary through llama.cpp.  This backend takes any object with
``tokenize``, ``detokenize`` and ``is_end_of_generation``; without one it works
on token ids only (``QwenIds``: Qwen2.5's end-of-generation ids, no text).
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from itertools import count

import torch

from .torch_model import PagedKVCache, PagedKVPool, TorchModel


@dataclass(frozen=True)
class StepOutput:
    """src/server/backend/base.py:5-8."""

    token: int
    finished: bool


class QwenIds:
    """Token-id-only vocabulary: <|endoftext|> (151643) and <|im_end|> (151645)
    end generation, as in Qwen2.5's vocabulary."""

    END_OF_GENERATION = frozenset({151643, 151645})

    def tokenize(self, text: str) -> list[int]:
        raise RuntimeError("no text vocabulary is attached; pass token ids")

    def detokenize(self, tokens: list[int]) -> bytes:
        raise RuntimeError("no text vocabulary is attached")

    def is_end_of_generation(self, token: int) -> bool:
        return token in self.END_OF_GENERATION


@dataclass
class _Sequence:
    cache: PagedKVCache
    pending: deque
    next_token: int | None = None  # the input of the next step, as an id or a token reference
    finished: bool = False
    feeds: object = None  # the launched step whose output the reference in next_token names


@dataclass
class LaunchedStep:
    """A step on the device: ``PagedBackend.finish`` turns it into outputs."""

    ids: object  # PendingTokens
    rows: list  # (seq_id, _Sequence, output row or None) per batch row


class PagedBackend:
    """src/server/backend/paged.py:21-99 with the model and pool on one GPU.

    ``num_blocks`` / ``block_size`` / ``prefill_chunk`` mean what they mean in
    the reference; ``max_seqs`` bounds the live sequences (device table rows).
    """

    def __init__(self, model: TorchModel, num_blocks: int, block_size: int, prefill_chunk: int,
                 vocab=None, max_seqs: int = 256, pool_dtype: torch.dtype | None = None):
        self._model = model
        max_blocks = min(num_blocks, -(-model.max_position // block_size))
        self._pool = PagedKVPool(model.config, num_blocks, block_size, device=model.device,
                                 dtype=pool_dtype or model.dtype, max_seqs=max_seqs,
                                 max_blocks_per_seq=max_blocks)
        self._num_blocks = num_blocks
        self._prefill_chunk = prefill_chunk
        self._vocab = vocab if vocab is not None else QwenIds()
        self._ids = count()
        self._sequences: dict[int, _Sequence] = {}

    @property
    def blocks_in_use(self) -> int:
        return self._num_blocks - self._pool.free_blocks

    @property
    def pool(self) -> PagedKVPool:
        return self._pool

    def tokenize(self, text: str) -> list[int]:
        return self._vocab.tokenize(text)

    def detokenize(self, tokens: list[int]) -> bytes:
        return self._vocab.detokenize(tokens)

    def start_sequence(self, prompt_tokens: list[int]) -> int:
        seq_id = next(self._ids)
        cache = self._pool.new_cache(seq_id)
        cache.reserve(0)
        self._sequences[seq_id] = _Sequence(cache, deque(prompt_tokens))
        return seq_id

    def step(self) -> dict[int, StepOutput]:
        launched = self.launch()
        return self.finish(launched) if launched is not None else {}

    def launch(self) -> LaunchedStep | None:
        """Composes and launches one step without waiting for it (the batch of
        ``step``).  A generating sequence whose last token has not reached the
        host yet feeds it by reference from the device, so the next step can be
        composed while this one runs; ``finish`` returns this step's outputs.
        A sequence that ends on an end-of-generation token revealed only by
        ``finish`` of the previous step still runs in this one: that row's
        output is dropped (``finish`` skips finished sequences)."""
        batch = self._generating_inputs() + self._prefill_inputs()
        if not batch:
            return None
        pending = self._model.launch_tokens(
            [(toks, self._sequences[s].cache) for s, toks in batch])
        rows = []
        for row, (seq_id, _) in enumerate(batch):
            sequence = self._sequences[seq_id]
            if sequence.pending:
                rows.append((seq_id, sequence, None))
            else:
                rows.append((seq_id, sequence, row))
        launched = LaunchedStep(pending, rows)
        for seq_id, sequence, row in rows:
            if row is not None:
                sequence.next_token = pending.ref(row)  # resolved on the device
                sequence.feeds = launched
        return launched

    def finish(self, launched: LaunchedStep) -> dict[int, StepOutput]:
        """Waits for a launched step: {seq_id: StepOutput} for every sequence
        whose prompt was fully consumed and that had not finished before."""
        tokens = launched.ids.result()
        outputs = {}
        for seq_id, sequence, row in launched.rows:
            if row is None or sequence.finished:
                continue
            token = tokens[row]
            if sequence.feeds is launched:
                sequence.next_token = token  # not relaunched yet: feed the id itself
                sequence.feeds = None
            sequence.finished = self._vocab.is_end_of_generation(token)
            outputs[seq_id] = StepOutput(token, sequence.finished)
        return outputs

    def release_sequence(self, seq_id: int) -> None:
        self._pool.release(self._sequences.pop(seq_id).cache)

    def close(self) -> None:
        pass

    def _generating_inputs(self) -> list[tuple[int, list[int]]]:
        return [
            (seq_id, [sequence.next_token])
            for seq_id, sequence in self._sequences.items()
            if not sequence.pending and not sequence.finished
        ]

    def _prefill_inputs(self) -> list[tuple[int, list[int]]]:
        inputs = []
        remaining = self._prefill_chunk
        for seq_id, sequence in self._sequences.items():
            take = min(remaining, len(sequence.pending))
            if take:
                inputs.append((seq_id, [sequence.pending.popleft() for _ in range(take)]))
                remaining -= take
        return inputs
