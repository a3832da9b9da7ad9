"""Host side of the engine's step graphs (no GPU): which padded graph serves a
step, and the int32 input vector that describes a step to it."""

import torch

from batchstream_inference_engine_b200.torch_model import ModelConfig, TorchModel, random_weights

TINY = ModelConfig(num_layers=1, hidden_size=32, num_heads=4, num_kv_heads=2, rope_theta=1e4,
                   rms_norm_eps=1e-6)


def tiny_model(**kw):
    weights = random_weights(TINY, vocab_size=50, intermediate_size=16)
    return TorchModel(TINY, weights, device="cpu", dtype=torch.float32, max_position=64, **kw)


def test_decode_buckets():
    m = tiny_model()
    assert [m._decode_bucket(n) for n in (0, 1, 2, 3, 5, 31, 32, 33, 100, 135, 256)] == \
        [0, 1, 2, 4, 8, 32, 32, 64, 128, 160, 256]
    assert m._graph_key([1] * 300) is None  # more decode rows than the largest graph


def test_graph_keys():
    m = tiny_model(max_graph_prefill=512, max_graph_chunks=8)
    assert m._graph_key([1, 1, 1]) == (4, 0, 0)
    assert m._graph_key([1] * 135 + [300, 212]) == (160, 2, 512)
    assert m._graph_key([7]) == (0, 1, 64)
    assert m._graph_key([1, 65]) == (1, 1, 128)
    assert m._graph_key([1, 5, 1]) == (1, 2, 64)  # a 1-token chunk after a chunk is a chunk
    assert m._graph_key([1, 513]) is None  # more prompt tokens than the largest graph
    assert m._graph_key([1] + [2] * 9) is None  # more chunks than the largest graph


def test_graph_inputs_layout():
    key = (4, 2, 64)  # B decode rows, P chunk rows, Q chunk tokens
    rows, starts, lengths = [7, 3, 9, 2], [10, 20, 0, 5], [1, 1, 3, 2]
    tokens = [[11], [12], [21, 22, 23], [31, 32]]
    v = TorchModel._graph_inputs(key, rows, starts, lengths, 2, tokens)
    B, P, Q = key
    R, T = B + P, B + Q
    assert len(v) == 3 * R + B + R + T
    seq_rows, start, n_new = v[:R], v[R:2 * R], v[2 * R:3 * R]
    after, ends, toks = v[3 * R:3 * R + B], v[3 * R + B:4 * R + B], v[4 * R + B:]
    assert seq_rows == [7, 3, 0, 0, 9, 2]
    assert start == [10, 20, -1, -1, 0, 5]  # padding rows start at -1
    assert n_new == [1, 1, 1, 1, 3, 2]  # every decode row (padding too) holds one token
    assert after == [11, 21, 0, 0]
    assert ends == [0, 1, 0, 0, 6, 8]  # chunk tokens start after the B decode tokens
    assert toks[:B] == [11, 12, 0, 0]
    assert toks[B:B + 5] == [21, 22, 23, 31, 32] and toks[B + 5:] == [0] * (Q - 5)


def test_graph_inputs_pads_chunk_rows():
    v = TorchModel._graph_inputs((1, 4, 64), [5, 6], [3, 0], [1, 4], 1, [[1], [2, 3, 4, 5]])
    R = 5
    assert v[R:2 * R] == [3, 0, -1, -1, -1]
    assert v[2 * R:3 * R] == [1, 4, 0, 0, 0]
    assert v[3 * R + 1:4 * R + 1] == [0, 4, 0, 0, 0]
