"""Workload definitions: the layer chains of the reference apps and of the benchmark configs,
their FLOP/byte counts, and seeded, chunk-deterministic synthetic data.

Conventions (the reference's perf.py scripts, e.g. apps/dlrm_topmlp/pipelined/perf.py:25):
  * FLOPs per row = 2 * sum(K_l * N_l) over the *logical* (unpadded) widths, GEMMs only.
  * Bytes per row = stored (padded) input row + output row (16-bit). Weights are read once per
    GPU and reported separately.

Data: inputs are generated on the host in fixed 65,536-row chunks, each from its own
torch.Generator seeded with (config seed, chunk index), so any row range (a GPU's shard, a
sample for the CPU oracle) can be regenerated identically anywhere. Weights come from one
generator per config. All values are rounded to the config's 16-bit type once; the oracle and the
kernels consume the same rounded numbers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import _lib as L

CHUNK_ROWS = 65536


@dataclass(frozen=True)
class Layer:
    k: int            # stored input width
    n: int            # output width
    act: int          # L.ACT_*
    k_logical: int    # unpadded input width (FLOP count)
    n_logical: int    # unpadded output width


@dataclass(frozen=True)
class Workload:
    name: str
    m: int
    dtype: torch.dtype
    layers: tuple
    tail: int = L.TAIL_NONE
    ln_eps: float = 1e-5
    seed: int = 0
    input_kind: str = "normal"    # normal | dlrm_dense | nerf_posenc
    input_logical: int = 0        # logical input columns (rest zero padding)
    weight_init: str = "kaiming"  # kaiming (nn.Linear default) | normal002 | xavier
    bias_init: str = "default"    # default (nn.Linear) | zero
    skip_layer: int = 0           # layer reading [previous output || x] (NeRF), 0 = none
    block: str = ""               # "" = one chain; "bert_addln" = attention-output Linear + x +
                                  # LN0, then the FFN chain (inputs: attn_out rows, then x rows);
                                  # "dlrm_interaction" = the DLRM feature interaction (inputs: m
                                  # bottom-output rows, then 26 m embedding rows; no layers);
                                  # "nerf_full" = NeRF with view directions (input: one flat
                                  # tensor, m x-rows of 64 then m d-rows of 32; output [m, 128]
                                  # holding out_r [m, 64] then out_rgb [m, 64] in memory order);
                                  # "mgn_mp" = one MeshGraphNet message-passing step over m edges
                                  # and m / 16 nodes (input: one flat fp16 buffer [ef | nf | srcs
                                  # | dsts], indices int64; output [m, 136] holding the edge rows
                                  # [m, 128] then the node rows [m / 16, 128])
    description: str = ""

    @property
    def k0(self) -> int:
        return self.layers[0].k

    @property
    def n_out(self) -> int:
        if self.block == "nerf_full":
            return 128
        if self.block == "mgn_mp":
            return 136
        return 480 if self.block == "dlrm_interaction" else self.layers[-1].n

    @property
    def widths(self) -> list:
        return [self.layers[0].k] + [l.n for l in self.layers]

    @property
    def acts(self) -> list:
        return [l.act for l in self.layers]

    @property
    def gp_dtype(self) -> int:
        return L.GP_BF16 if self.dtype == torch.bfloat16 else L.GP_F16

    @property
    def flop_per_row(self) -> int:
        if self.block == "dlrm_interaction":
            return 351 * 2 * 128  # the dot products below the diagonal
        if self.block == "mgn_mp":  # edge MLP per edge, node MLP per 16 edges
            e = sum(2 * l.k_logical * l.n_logical for l in self.layers[:3])
            return e + sum(2 * l.k_logical * l.n_logical for l in self.layers[3:]) // MGN_EDGES_PER_NODE
        return sum(2 * l.k_logical * l.n_logical for l in self.layers)

    @property
    def in_width(self) -> int:
        """Stored input bytes per row / 2 (attn_out and x for the bert_addln block)."""
        if self.block == "dlrm_interaction":
            return 27 * 128
        if self.block.startswith("nerf_full"):
            return 96
        if self.block == "mgn_mp":
            return 128 + 8 + 8  # ef, nf / 16, two int64 indices
        return 2 * self.k0 if self.block == "bert_addln" else self.k0

    @property
    def bytes_per_row(self) -> int:
        return 2 * (self.in_width + self.n_out)

    @property
    def n_out_logical(self) -> int:
        return self.layers[-1].n_logical

    @property
    def weight_bytes(self) -> int:
        b = sum(2 * (l.k * l.n + l.n) for l in self.layers)
        if self.tail != L.TAIL_NONE:
            b += 4 * self.n_out
        return b

    def spec(self) -> L.GpSpec:
        return L.make_spec(self.widths, self.acts, self.tail, self.gp_dtype, self.ln_eps,
                           self.skip_layer)

    @property
    def bound(self) -> str:
        """'hbm' or 'tensor': the slower of FLOPs at the bf16 peak and bytes at HBM bandwidth
        (ridge of the measured peaks, about 253 FLOP/B)."""
        return "tensor" if self.flop_per_row / self.bytes_per_row > 253 else "hbm"

    def with_m(self, m: int) -> "Workload":
        return Workload(**{**self.__dict__, "m": int(m)})


def _mgn(name, m, k0, seed, tail=L.TAIL_LAYERNORM, dtype=torch.float16, desc=""):
    R, N = L.ACT_RELU, L.ACT_NONE
    return Workload(
        name=name, m=m, dtype=dtype, seed=seed, tail=tail, ln_eps=1e-5,
        layers=(Layer(k0, 128, R, k0, 128), Layer(128, 128, R, 128, 128), Layer(128, 128, N, 128, 128)),
        input_logical=k0, description=desc)


# Benchmark configs (the reference's MeshGraphNet MLP, common/mlps.py:3-20 MgnMlp(k0, [128]*3))
MGN_EDGE = _mgn("mgn_edge", 65536, 384, 0,
                desc="MeshGraphNet edge MLP: 384->128 ReLU->128 ReLU->128, LayerNorm(128), fp16")
MGN_NODE = _mgn("mgn_node", 1048576, 256, 1,
                desc="MeshGraphNet node MLP: 256->128 ReLU->128 ReLU->128, LayerNorm(128), fp16")

# Reference apps served by the same kernel family
MGN_LINEARS = _mgn("mgn_linears", 1310720, 384, 0, tail=L.TAIL_NONE,
                   desc="apps/mgn_linears: 384->128->128->128 without LayerNorm")
TEST_MLP = _mgn("test_mlp", 1310720, 128, 0, tail=L.TAIL_NONE,
                desc="apps/test_mlp: 128->128->128->128")

# DLRM bottom MLP (common/mlps.py:23-35 DlrmMlp([13, 512, 256, 128])): 13 dense features padded
# to 16; Xavier-uniform weights (seed 3); ReLU after every layer.
_R, _N = L.ACT_RELU, L.ACT_NONE
DLRM_BOT = Workload(
    name="dlrm_bot", m=262144, dtype=torch.float16, seed=3, input_kind="dlrm_dense",
    input_logical=13, weight_init="xavier",
    layers=(Layer(16, 512, _R, 13, 512), Layer(512, 256, _R, 512, 256), Layer(256, 128, _R, 256, 128)),
    description="DLRM bottom MLP: 13(16)->512->256->128, ReLU, fp16")

# GraphCast-style edge MLP (apps/gc_edges/torch/model.py with SiLU): bf16, seed 4.
GC_EDGE = Workload(
    name="gc_edge", m=1638400, dtype=torch.bfloat16, seed=4, tail=L.TAIL_LAYERNORM, ln_eps=1e-5,
    input_logical=1536,
    layers=(Layer(1536, 512, L.ACT_SILU, 1536, 512), Layer(512, 512, _N, 512, 512)),
    description="GraphCast edge MLP: 1536->512 SiLU->512, LayerNorm(512), bf16")

# NeRF MLP (apps/nerf_full/torch/model.py, use_viewdirs=False, out_ch=4): positional encoding of
# xyz ~ U(-1, 1), 63 features padded to 64; skip concat of x into layer 5; 256 -> 4 head.
NERF = Workload(
    name="nerf", m=4194304, dtype=torch.float16, seed=4, input_kind="nerf_posenc", input_logical=63,
    skip_layer=5,
    layers=(Layer(64, 256, _R, 63, 256),) + tuple(Layer(256, 256, _R, 256, 256) for _ in range(4)) +
           (Layer(320, 256, _R, 319, 256), Layer(256, 256, _R, 256, 256), Layer(256, 256, _R, 256, 256),
            Layer(256, 4, _N, 256, 4)),
    description="NeRF MLP: 63(64)->256 x5, [h||x] 319(320)->256, 256 x2, ReLU, 256->4 head, fp16")

# BERT-large FFN (apps/bert_ffn/torch/model.py at H=1024, ff=4096, GELU(tanh), LN eps 1e-12):
# weights N(0, 0.02^2), zero biases, seed 2, bf16.
BERT_FFN = Workload(
    name="bert_ffn", m=16384, dtype=torch.bfloat16, seed=2, tail=L.TAIL_RESIDUAL_LN, ln_eps=1e-12,
    input_logical=1024, weight_init="normal002", bias_init="zero",
    layers=(Layer(1024, 4096, L.ACT_GELU_TANH, 1024, 4096), Layer(4096, 1024, _N, 4096, 1024)),
    description="BERT-large FFN: 1024->4096 GELU->1024, +x, LayerNorm(1024, 1e-12), bf16")

# DLRM top MLP (DlrmMlp([479, 1024, 1024, 512, 256, 1], sigmoid_i=4)): input 479 padded to 480
# (the 128-wide bottom output concatenated with 351 interaction values); Xavier-uniform, seed 3.
DLRM_TOP = Workload(
    name="dlrm_top", m=262144, dtype=torch.float16, seed=3, input_logical=479, weight_init="xavier",
    layers=(Layer(480, 1024, _R, 479, 1024), Layer(1024, 1024, _R, 1024, 1024),
            Layer(1024, 512, _R, 1024, 512), Layer(512, 256, _R, 512, 256),
            Layer(256, 1, L.ACT_SIGMOID, 256, 1)),
    description="DLRM top MLP: 479(480)->1024->1024->512->256 ReLU ->1 sigmoid, fp16")

# BERT attention-output block (apps/bert_addln_ffn, model.py:4-19) at the reference's widths and
# row count (perf.py: M = 64 * 512): h = LN0(attn_out W0 + b0 + x), LN2(FFN(h) + h), fp16, ReLU.
BERT_ADDLN = Workload(
    name="bert_addln", m=32768, dtype=torch.float16, seed=5, tail=L.TAIL_RESIDUAL_LN, ln_eps=1e-5,
    input_logical=128, block="bert_addln",
    layers=(Layer(128, 128, _N, 128, 128), Layer(128, 512, _R, 128, 512), Layer(512, 128, _N, 512, 128)),
    description="BERT attention-output block: 128->128 +x LN0, 128->512 ReLU->128 +h LN2, fp16")

# DLRM feature interaction between the bottom and top MLPs (graphmodel/dlrm.py:28-42) at the DLRM
# batch: bottom outputs (ReLU-like, >= 0) and 26 embedding vectors per sample, fp16.
DLRM_INTERACT = Workload(
    name="dlrm_interact", m=262144, dtype=torch.float16, seed=6, block="dlrm_interaction",
    layers=(Layer(128, 480, _N, 128, 480),), input_logical=128,
    description="DLRM interaction: [bot; 26 embeddings] (27 x 128) -> bot | 351 dot products | 0 (480), fp16")

# NeRF with view directions (apps/nerf_full, model.py:40-64 with use_viewdirs=True) at the
# reference's pipelined shapes (nerf_full_pl_ext.cu:54-66: x 64, d 32, alpha and rgb padded to
# 64): trunk as NERF, alpha 256 -> 64, bottleneck 256 -> 256, rgb [bottleneck | d] 288 -> 128 ReLU
# -> 64. x is the 63-feature positional encoding (padded to 64); d the 27-feature encoding of a
# unit view direction (direction + 4 octaves of sin/cos), padded to 32. Layer list = w1..w12.
NERF_FULL = Workload(
    name="nerf_full", m=1048576, dtype=torch.float16, seed=8, input_kind="nerf_posenc",
    input_logical=63, skip_layer=5, block="nerf_full",
    layers=(Layer(64, 256, _R, 63, 256),) + tuple(Layer(256, 256, _R, 256, 256) for _ in range(4)) +
           (Layer(320, 256, _R, 319, 256), Layer(256, 256, _R, 256, 256), Layer(256, 256, _R, 256, 256),
            Layer(256, 64, _N, 256, 64), Layer(256, 256, _N, 256, 256), Layer(288, 128, _R, 283, 128),
            Layer(128, 64, _N, 128, 64)),
    description="NeRF with view directions: trunk 63(64)->256 x8 (skip), alpha 256->64, "
                "bottleneck 256->256, rgb [256 | d 27(32)] -> 128 ReLU -> 64, fp16")

# One MeshGraphNet message-passing step (graphmodel/mgn_dp.py:28-54, one edge set): edge update
# [nf[src] | ef | nf[dst]] -> MgnMlp(384) + LN with the gather and the segment sum by destination
# fused, then the node update [nf | aggregate] -> MgnMlp(256) + LN. 16 edges per node (the ratio of
# mgn_dp.py's mesh edges to nodes); endpoints uniform over the nodes; features ~N(0, 1).
MGN_EDGES_PER_NODE = 16
MGN_MP = Workload(
    name="mgn_mp", m=2097152, dtype=torch.float16, seed=9, tail=L.TAIL_LAYERNORM, ln_eps=1e-5,
    input_logical=384, block="mgn_mp",
    layers=(Layer(384, 128, _R, 384, 128), Layer(128, 128, _R, 128, 128), Layer(128, 128, _N, 128, 128),
            Layer(256, 128, _R, 256, 128), Layer(128, 128, _R, 128, 128), Layer(128, 128, _N, 128, 128)),
    description="MeshGraphNet message passing: edges [nf[src] | ef | nf[dst]] 384->128->128->128 + LN "
                "(gather and segment sum fused), nodes [nf | agg] 256->128->128->128 + LN, 16 edges "
                "per node, fp16")

WORKLOADS = {w.name: w for w in (MGN_EDGE, MGN_NODE, MGN_LINEARS, TEST_MLP, DLRM_BOT, GC_EDGE, NERF,
                                 BERT_FFN, DLRM_TOP, BERT_ADDLN, DLRM_INTERACT, NERF_FULL, MGN_MP)}


def rows_of(w: Workload, x: torch.Tensor) -> int:
    """Rows of workload input `x` (the bert_addln block stacks attn_out rows over x rows)."""
    if w.block == "dlrm_interaction":
        return x.shape[0] // 27
    if w.block == "nerf_full":
        return x.numel() // 96
    if w.block == "mgn_mp":
        return x.numel() // w.in_width
    return x.shape[0] // 2 if w.block == "bert_addln" else x.shape[0]


# ------------------------------------------------------------------------------------------------
# seeded data
# ------------------------------------------------------------------------------------------------
def _gen(seed: int, *salt: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    s = seed
    for v in salt:
        s = (s * 1000003 + v + 0x9E3779B1) % (2**63 - 1)
    g.manual_seed(s)
    return g


def make_weights(w: Workload):
    """Per layer: (W [k, n] in w.dtype, b [n] in w.dtype); plus (gamma, beta) for LN tails.

    Weights use the [K, N] layout the reference's C++ kernels take (`weight.t().contiguous()`).
    Padded input rows/columns (stored k > logical k) are zero.
    """
    if w.block == "dlrm_interaction":
        return [], None
    g = _gen(w.seed, 7777)
    layers = []
    for l in w.layers:
        kl, nl = l.k_logical, l.n_logical
        if w.weight_init == "kaiming":
            bound = 1.0 / math.sqrt(kl)   # nn.Linear default: kaiming_uniform(a=sqrt(5))
            wt = (torch.rand(nl, kl, generator=g) * 2 - 1) * bound
        elif w.weight_init == "normal002":
            wt = torch.randn(nl, kl, generator=g) * 0.02
        elif w.weight_init == "xavier":
            bound = math.sqrt(6.0 / (kl + nl))
            wt = (torch.rand(nl, kl, generator=g) * 2 - 1) * bound
        else:
            raise ValueError(w.weight_init)
        if w.bias_init == "zero":
            bt = torch.zeros(nl)
        else:
            bt = (torch.rand(nl, generator=g) * 2 - 1) / math.sqrt(kl)
        W = torch.zeros(l.k, l.n)
        W[:kl, :nl] = wt.t()
        B = torch.zeros(l.n)
        B[:nl] = bt
        layers.append((W.to(w.dtype).contiguous(), B.to(w.dtype).contiguous()))
    ln = None
    if w.tail != L.TAIL_NONE:
        nl = w.layers[-1].n
        ln = (torch.ones(nl, dtype=w.dtype), torch.zeros(nl, dtype=w.dtype))
        if w.block in ("bert_addln", "mgn_mp"):  # two LayerNorms (LN0 / LN2, edge / node)
            ln = ln + (torch.ones(nl, dtype=w.dtype), torch.zeros(nl, dtype=w.dtype))
    return layers, ln


def make_input_chunk(w: Workload, chunk: int, rows: int | None = None) -> torch.Tensor:
    """Rows [chunk*CHUNK_ROWS, chunk*CHUNK_ROWS + rows) of the input, in w.dtype."""
    rows = CHUNK_ROWS if rows is None else rows
    g = _gen(w.seed, 1, chunk)
    if w.block == "mgn_mp":
        return mgn_graph_input(w, rows, chunk)
    if w.block == "dlrm_interaction":
        # [bottom-output rows (ReLU of N(0, 0.3^2)); 26 embedding rows per sample, N(0, 0.1^2)]
        bot = torch.relu(torch.randn(rows, w.k0, generator=g)) * 0.3
        emb = torch.randn(rows * 26, w.k0, generator=_gen(w.seed, 2, chunk)) * 0.1
        return torch.cat([bot, emb]).to(w.dtype)
    if w.block == "bert_addln":
        # [attn_out rows; x rows], both ~N(0, 1)
        return torch.cat([torch.randn(rows, w.k0, generator=g),
                          torch.randn(rows, w.k0, generator=_gen(w.seed, 2, chunk))]).to(w.dtype)
    if w.input_kind == "normal":
        x = torch.randn(rows, w.k0, generator=g)
    elif w.input_kind == "dlrm_dense":
        # log1p of Exp(1) draws (DLRM's dense-feature transform)
        x = torch.log1p(torch.empty(rows, w.k0).exponential_(1.0, generator=g))
    elif w.input_kind == "nerf_posenc" and w.block.startswith("nerf_full"):
        x = _nerf_posenc(torch.rand(rows, 3, generator=g) * 2 - 1, 10, 64)
        v = torch.randn(rows, 3, generator=_gen(w.seed, 2, chunk))
        d = _nerf_posenc(v / v.norm(dim=1, keepdim=True).clamp_min(1e-6), 4, 32)
        xd = torch.cat([x, d], dim=1).to(w.dtype)  # [rows, 96]
        if w.block == "nerf_full":
            return torch.cat([xd[:, :64].reshape(-1), xd[:, 64:].reshape(-1)])
        return xd
    elif w.input_kind == "nerf_posenc":
        # gamma(p) = [p, sin(2^k pi p), cos(2^k pi p)]_{k=0..9} for xyz ~ U(-1, 1)
        p = torch.rand(rows, 3, generator=g) * 2 - 1
        feats = [p]
        for k in range(10):
            feats += [torch.sin((2.0 ** k) * math.pi * p), torch.cos((2.0 ** k) * math.pi * p)]
        x = torch.zeros(rows, w.k0)
        x[:, :63] = torch.cat(feats, dim=1)
    else:
        raise ValueError(w.input_kind)
    if w.input_logical < w.k0:
        x[:, w.input_logical:] = 0
    return x.to(w.dtype)


def _nerf_posenc(p: torch.Tensor, octaves: int, width: int) -> torch.Tensor:
    """[p, sin(2^k pi p), cos(2^k pi p)]_{k < octaves}, zero-padded to `width` columns."""
    feats = [p]
    for k in range(octaves):
        feats += [torch.sin((2.0 ** k) * math.pi * p), torch.cos((2.0 ** k) * math.pi * p)]
    f = torch.cat(feats, dim=1)
    out = torch.zeros(p.shape[0], width)
    out[:, :f.shape[1]] = f
    return out


def mgn_graph_input(w: Workload, edges: int, salt: int) -> torch.Tensor:
    """A graph of `edges` edges and edges / 16 nodes, packed as one flat fp16 buffer:
    [ef (edges x 128) | nf (nodes x 128) | srcs (int64) | dsts (int64)]."""
    assert edges % MGN_EDGES_PER_NODE == 0, "edges must be a multiple of 16"
    nodes = edges // MGN_EDGES_PER_NODE
    g = _gen(w.seed, 3, salt)
    ef = torch.randn(edges, 128, generator=g).to(w.dtype)
    nf = torch.randn(nodes, 128, generator=g).to(w.dtype)
    idx = torch.randint(0, nodes, (2, edges), generator=g)
    return torch.cat([ef.reshape(-1), nf.reshape(-1), idx.reshape(-1).view(w.dtype)])


def split_mgn_input(x: torch.Tensor):
    """Inverse of mgn_graph_input: (ef, nf, srcs, dsts) views of the flat buffer."""
    edges = x.numel() // 144
    nodes = edges // MGN_EDGES_PER_NODE
    ef = x[:edges * 128].view(edges, 128)
    nf = x[edges * 128:(edges + nodes) * 128].view(nodes, 128)
    idx = x[(edges + nodes) * 128:].view(torch.int64).view(2, edges)
    return ef, nf, idx[0], idx[1]


def make_input(w: Workload, row0: int = 0, rows: int | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows [row0, row0+rows) of the input (host tensor, optionally written into `out`)."""
    rows = w.m - row0 if rows is None else rows
    if w.block == "dlrm_interaction":
        bots, embs = [], []
        r = row0
        while r < row0 + rows:
            c = r // CHUNK_ROWS
            c0 = c * CHUNK_ROWS
            take = min(c0 + CHUNK_ROWS, row0 + rows) - r
            need = r - c0 + take
            chunk = make_input_chunk(w, c, need)
            bots.append(chunk[r - c0:r - c0 + take])
            embs.append(chunk[need + 26 * (r - c0):need + 26 * (r - c0 + take)])
            r += take
        res = torch.cat(bots + embs) if rows else torch.empty(0, w.k0, dtype=w.dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res
    if w.block == "bert_addln":
        a = torch.empty(rows, w.k0, dtype=w.dtype)
        b = torch.empty(rows, w.k0, dtype=w.dtype)
        r = row0
        while r < row0 + rows:
            c = r // CHUNK_ROWS
            c0 = c * CHUNK_ROWS
            take = min(c0 + CHUNK_ROWS, row0 + rows) - r
            need = r - c0 + take
            chunk = make_input_chunk(w, c, need)
            a[r - row0:r - row0 + take] = chunk[r - c0:r - c0 + take]
            b[r - row0:r - row0 + take] = chunk[need + r - c0:need + r - c0 + take]
            r += take
        res = torch.cat([a, b])
        if out is not None:
            out.copy_(res)
            return out
        return res
    if w.block == "mgn_mp":
        # each rank / sample is its own graph (message passing does not split a graph by rows here)
        res = mgn_graph_input(w, rows, row0 // MGN_EDGES_PER_NODE)
        if out is not None:
            out.copy_(res)
            return out
        return res
    if w.block == "nerf_full":
        res = make_input(Workload(**{**w.__dict__, "block": "nerf_full_rows"}), row0, rows)
        flat = torch.cat([res[:, :64].reshape(-1), res[:, 64:].reshape(-1)])
        if out is not None:
            out.copy_(flat)
            return out
        return flat
    if out is None:
        out = torch.empty(rows, w.in_width if w.block == "nerf_full_rows" else w.k0, dtype=w.dtype)
    r = row0
    while r < row0 + rows:
        c = r // CHUNK_ROWS
        c0 = c * CHUNK_ROWS
        take = min(c0 + CHUNK_ROWS, row0 + rows) - r
        need = r - c0 + take
        chunk = make_input_chunk(w, c, need)
        out[r - row0:r - row0 + take] = chunk[r - c0:r - c0 + take]
        r += take
    return out


def shard_rows(m: int, world: int, rank: int, tile: int = 128) -> tuple:
    """Contiguous row range of `rank`: ceil(m / world) rounded up to the tile, tail on the last."""
    per = -(-m // world)
    per = -(-per // tile) * tile
    r0 = min(rank * per, m)
    r1 = min(r0 + per, m)
    return r0, r1 - r0
