"""CPU tests of the tensor-parallel partition (q38cu_tp_shard, host only).

The shards must cover every head, FFN block and vocabulary row exactly once;
a shard's local DeltaNet value heads must read their key heads through the
kernel's local rule (local key head = local value head % local key heads,
the image of the upstream's key_head = value_head % 16,
qwen38_model.c:764); attention query heads must find their KV heads
(kv_head = head / 6, qwen38_model.c:851).  Then two gloo ranks (CPU
processes) run the row-parallel projections of the plan on quantized weights
with the upstream Q8_K kernels (oracle): each rank's partial over its input
superblocks, summed by an all-reduce, must equal the full projection.
"""
import os
import socket

import numpy as np
import pytest

from q38b200.model import tp_shard

WORLDS = (1, 2, 4, 8)


def shards(world):
    return [tp_shard(r, world) for r in range(world)]


@pytest.mark.parametrize("world", WORLDS)
def test_shards_cover_the_model_once(world):
    ss = shards(world)
    keys = sorted(k for s in ss for k in s.key_heads[:s.n_key_heads])
    blocks = sorted(b for s in ss for b in s.value_blocks[:s.n_value_blocks])
    assert keys == list(range(16)) and blocks == list(range(24))
    heads = sorted(h for s in ss for h in range(s.attn_head0, s.attn_head0 + s.attn_heads))
    assert heads == list(range(24))
    ffn = sorted(i for s in ss for i in range(s.ffn0 // 256, (s.ffn0 + s.ffn) // 256))
    assert ffn == list(range(68)) and all(s.ffn0 % 256 == 0 and s.ffn % 256 == 0 for s in ss)
    vocab = sorted((s.vocab0, s.vocab0 + s.vocab) for s in ss)
    assert vocab[0][0] == 0 and vocab[-1][1] == 248320
    assert all(a[1] == b[0] for a, b in zip(vocab, vocab[1:]))
    assert len({s.vocab for s in ss}) == 1, "all-gather needs equal slices"


@pytest.mark.parametrize("world", WORLDS)
def test_local_heads_read_their_key_and_kv_heads(world):
    for s in shards(world):
        n_kh = s.n_key_heads
        keys = list(s.key_heads[:n_kh])
        for local_v in range(2 * s.n_value_blocks):
            global_v = 2 * s.value_blocks[local_v // 2] + local_v % 2
            assert keys[local_v % n_kh] == global_v % 16, (s.rank, local_v)
        for h in range(s.attn_head0, s.attn_head0 + s.attn_heads):
            assert s.kv_head0 <= h // 6 < s.kv_head0 + s.kv_heads


def test_bad_partitions_are_refused():
    from q38b200.model import ModelError
    for rank, world in ((0, 3), (2, 2), (0, 16)):
        with pytest.raises(ModelError):
            tp_shard(rank, world)


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _gather_cols(data, qtype, rows, width, block_ranges):
    """Rows of a GGUF tensor restricted to the listed superblock ranges."""
    import oracle as O
    row_bytes = O.row_bytes(qtype, width)
    bb = O.BLOCK[qtype][1]
    rows_view = np.asarray(data, np.uint8).reshape(rows, row_bytes)
    return np.concatenate([rows_view[:, b0 * bb:b1 * bb] for b0, b1 in block_ranges], axis=1)


def _rank_main(rank, world, port, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "qwen3.8-27b-in-c_b200", "python")]
    import torch
    import torch.distributed as dist
    import oracle as O
    from q38b200 import synth
    from q38b200.model import tp_shard as shard_of
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    ref = O.Oracle()
    s = shard_of(rank, world)
    rows = 5120
    results = {}
    # ssm_out: input superblocks = this rank's DeltaNet output blocks, in local order
    w = synth.quant_tensor(O.Q4_K, rows, 6144, seed=11)
    x = synth.activations(1, 6144, seed=12)
    blocks = [int(b) for b in s.value_blocks[:s.n_value_blocks]]
    local_w = _gather_cols(w, O.Q4_K, rows, 6144, [(b, b + 1) for b in blocks])
    local_x = np.concatenate([x[:, 256 * b:256 * b + 256] for b in blocks], axis=1)
    part = ref.gemm_q8_k(O.Q4_K, local_w, rows, local_x.shape[1], ref.quantize_q8_k(local_x))
    # ffn_down (Q6_K): input superblocks = this rank's FFN blocks
    wd = synth.quant_tensor(O.Q6_K, rows, 17408, seed=13)
    xd = synth.activations(1, 17408, seed=14)
    b0, b1 = s.ffn0 // 256, (s.ffn0 + s.ffn) // 256
    local_wd = _gather_cols(wd, O.Q6_K, rows, 17408, [(b0, b1)])
    part_d = ref.gemm_q8_k(O.Q6_K, local_wd, rows, s.ffn, ref.quantize_q8_k(xd[:, 256 * b0:256 * b1]))
    for name, p in (("ssm_out", part), ("ffn_down", part_d)):
        t = torch.from_numpy(np.ascontiguousarray(p, np.float32))
        dist.all_reduce(t)
        results[name] = t.numpy()
    if rank == 0:
        np.savez(os.path.join(out_dir, "reduced.npz"), **results)
    dist.destroy_process_group()


def test_row_parallel_projections_sum_to_the_whole(tmp_path, oracle):
    """Two gloo ranks: the partial ssm_out and ffn_down products over each
    rank's input superblocks, all-reduced, equal the whole projections (the
    Q8_K activation blocks of a slice are the whole activation's blocks)."""
    import torch.multiprocessing as mp
    import oracle as O
    from q38b200 import synth
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    got = np.load(os.path.join(tmp_path, "reduced.npz"))
    rows = 5120
    w = synth.quant_tensor(O.Q4_K, rows, 6144, seed=11)
    x = synth.activations(1, 6144, seed=12)
    want = oracle.gemm_q8_k(O.Q4_K, w, rows, 6144, oracle.quantize_q8_k(x))
    np.testing.assert_allclose(got["ssm_out"], want, rtol=1e-4, atol=1e-4 * np.abs(want).max())
    wd = synth.quant_tensor(O.Q6_K, rows, 17408, seed=13)
    xd = synth.activations(1, 17408, seed=14)
    want_d = oracle.gemm_q8_k(O.Q6_K, wd, rows, 17408, oracle.quantize_q8_k(xd))
    np.testing.assert_allclose(got["ffn_down"], want_d, rtol=1e-4, atol=1e-4 * np.abs(want_d).max())
