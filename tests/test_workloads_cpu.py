"""Host logic: FLOP/byte accounting, chunk-deterministic data, row sharding."""
import torch

from gpu_pipes_b200 import workloads as W


def test_flops_and_bytes_match_baseline_table():
    assert W.MGN_EDGE.flop_per_row == 163840
    assert W.MGN_EDGE.bytes_per_row == 1024
    assert W.MGN_NODE.flop_per_row == 131072
    assert W.MGN_NODE.bytes_per_row == 768


def test_input_rows_are_chunk_deterministic():
    w = W.MGN_NODE.with_m(200000)
    full = W.make_input(w, 0, 140000)
    part = W.make_input(w, 65000, 70000)
    assert torch.equal(full[65000:135000], part)
    again = W.make_input(w, 131000, 1000)
    assert torch.equal(full[131000:132000], again)


def test_weights_deterministic():
    a, _ = W.make_weights(W.MGN_EDGE)
    b, _ = W.make_weights(W.MGN_EDGE)
    for (wa, ba), (wb, bb) in zip(a, b):
        assert torch.equal(wa, wb) and torch.equal(ba, bb)
    assert a[0][0].shape == (384, 128) and a[0][0].dtype == torch.float16


def test_shard_rows_cover_exactly():
    for m in (1, 127, 65536, 1048576, 1000003):
        for world in (1, 2, 4, 8):
            got = []
            for r in range(world):
                r0, n = W.shard_rows(m, world, r)
                assert n >= 0
                if n:
                    assert r0 % 128 == 0
                got.append((r0, n))
            covered = sum(n for _, n in got)
            assert covered == m
            pos = 0
            for r0, n in got:
                if n:
                    assert r0 == pos
                    pos += n
