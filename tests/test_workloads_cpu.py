"""Host logic: FLOP/byte accounting, chunk-deterministic data, row sharding."""
import torch

from gpu_pipes_b200 import workloads as W
from oracle import mlp_oracle as O


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


def test_mgn_mp_packing_round_trip():
    """The mgn_mp input is one flat fp16 buffer [ef | nf | srcs | dsts]; split_mgn_input recovers
    the parts, indices in range, and the oracle step sums each edge into its destination."""
    w = W.WORKLOADS["mgn_mp"]
    x = W.make_input(w, 0, 4096)
    assert x.dtype == torch.float16 and x.dim() == 1 and W.rows_of(w, x) == 4096
    ef, nf, srcs, dsts = W.split_mgn_input(x)
    assert ef.shape == (4096, 128) and nf.shape == (256, 128)
    assert srcs.dtype == torch.int64 and int(srcs.min()) >= 0 and int(srcs.max()) < 256
    assert int(dsts.min()) >= 0 and int(dsts.max()) < 256
    assert torch.equal(x, W.make_input_chunk(w, 0, 4096))
    layers, ln = W.make_weights(w)
    assert len(layers) == 6 and len(ln) == 4
    y = O.workload_forward(w, x, layers, ln)
    assert y.shape == (4096, 136)
    flat = y.reshape(-1)
    y_e = flat[:4096 * 128].view(4096, 128)
    agg = O.mgn_aggregate(y_e.half(), dsts, 256)
    y_n = O.mgn_node_update(nf, [agg], layers[3:], (ln[2], ln[3]))
    torch.testing.assert_close(flat[4096 * 128:].view(256, 128), y_n)


def test_nerf_full_input_layout():
    """The nerf_full input is [x rows (M x 64) | d rows (M x 32)], row ranges consistent across
    chunk boundaries; d rows are unit-direction encodings (first 3 columns of norm 1)."""
    w = W.WORKLOADS["nerf_full"]
    a = W.make_input(w, 65500, 100)
    full = W.make_input(w, 65400, 300)
    m = 300
    x_full, d_full = full[:m * 64].view(m, 64), full[m * 64:].view(m, 32)
    x_a, d_a = a[:100 * 64].view(100, 64), a[100 * 64:].view(100, 32)
    assert torch.equal(x_a, x_full[100:200]) and torch.equal(d_a, d_full[100:200])
    norms = d_full[:, :3].float().norm(dim=1)
    assert torch.allclose(norms, torch.ones_like(norms), atol=2e-3)
    assert torch.all(d_full[:, 27:] == 0) and torch.all(x_full[:, 63:] == 0)


def test_mgn_mp_rank_graphs_distinct_and_reproducible():
    """Under weak scaling each rank builds its own graph from its row offset: the same rank gets
    the same bytes, different ranks different graphs."""
    w = W.WORKLOADS["mgn_mp"].with_m(4096)
    g0 = W.make_input(w.with_m(4096), 0, 4096)
    g1 = W.make_input(w.with_m(2 * 4096), 4096, 4096)
    assert torch.equal(g0, W.make_input(w.with_m(4096), 0, 4096))
    assert torch.equal(g1, W.make_input(w.with_m(2 * 4096), 4096, 4096))
    assert not torch.equal(g0, g1)
