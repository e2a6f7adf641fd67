"""Host side of the batched prefill, on the CPU: how prompts are split into chunks and how one
chunk's metadata (token rows, positions, context lengths, block tables per row and per sequence,
the attention tile order) is packed into the single int32 buffer the kernels read.  The reference
prefills one sequence at a time (``mini_vllm/engine/engine.py:253-295``): row r of a chunk is
token i of sequence s at position i, exactly what that per-sequence pass feeds its model."""
import pytest
import torch

from llm_pytorch_inference_b200.prefill import pack_chunk_metadata, split_chunks


def test_split_chunks_takes_whole_sequences_greedily():
    assert split_chunks([5, 10, 3, 7], 15) == [(0, 2), (2, 4)]
    assert split_chunks([5, 10, 3, 7], 25) == [(0, 4)]
    assert split_chunks([15, 15, 1], 15) == [(0, 1), (1, 2), (2, 3)]   # exact fits
    assert split_chunks([], 8) == []
    with pytest.raises(ValueError, match="exceeds the prefill budget"):
        split_chunks([4, 20, 1], 16)


def test_pack_chunk_metadata_layout():
    ids = [[1, 2, 3], list(range(100, 117)), [9]]          # 3, 17 and 1 tokens
    tables = [[7], [3, 5], [11]]
    mb, scratch = 3, 99
    host, (T, S, nt, o_seq, o_tile) = pack_chunk_metadata(ids, tables, mb, scratch)
    assert (T, S, nt) == (21, 3, 4)
    assert host.dtype == torch.int32 and host.numel() == o_tile + 2 * nt
    assert o_seq == 3 * T + T * mb and o_tile == o_seq + 2 * S + S * mb
    tok, pos, ctx = host[:T], host[T:2 * T], host[2 * T:3 * T]
    assert tok.tolist() == [1, 2, 3] + list(range(100, 117)) + [9]
    assert pos.tolist() == [0, 1, 2] + list(range(17)) + [0]
    assert torch.equal(ctx, pos + 1)
    bt = host[3 * T:o_seq].view(T, mb)
    assert bt[:3].tolist() == [[7, 99, 99]] * 3
    assert bt[3:20].tolist() == [[3, 5, 99]] * 17
    assert bt[20].tolist() == [11, 99, 99]
    assert host[o_seq:o_seq + S].tolist() == [0, 3, 20]               # sequence starts
    assert host[o_seq + S:o_seq + 2 * S].tolist() == [3, 17, 1]       # sequence lengths
    assert host[o_seq + 2 * S:o_tile].view(S, mb).tolist() == [[7, 99, 99], [3, 5, 99], [11, 99, 99]]
    # tiles (sequence, 16-token query tile): the second tile of the 17-token prompt first (longest
    # prefix), then the first tiles in sequence order
    assert host[o_tile:o_tile + nt].tolist() == [1, 0, 1, 2]
    assert host[o_tile + nt:].tolist() == [1, 0, 0, 0]


def test_pack_chunk_metadata_rejects_a_table_wider_than_max_blocks():
    with pytest.raises(ValueError, match="max_blocks"):
        pack_chunk_metadata([[1] * 40], [[1, 2, 3]], 2, 0)


def test_tile_order_puts_longer_prefixes_first():
    lens = [50, 200, 16, 33]
    ids = [[0] * n for n in lens]
    tables = [list(range((n + 15) // 16)) for n in lens]
    host, (T, S, nt, o_seq, o_tile) = pack_chunk_metadata(ids, tables, 13, 0)
    seq = host[o_tile:o_tile + nt].tolist()
    idx = host[o_tile + nt:].tolist()
    assert nt == sum((n + 15) // 16 for n in lens)
    assert sorted(zip(seq, idx)) == sorted((s, q) for s, n in enumerate(lens) for q in range((n + 15) // 16))
    assert idx == sorted(idx, reverse=True)
    for k in range(1, nt):   # stable: equal tile indices keep sequence order
        if idx[k] == idx[k - 1]:
            assert seq[k] > seq[k - 1]
