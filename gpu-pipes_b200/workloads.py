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
    description: str = ""

    @property
    def k0(self) -> int:
        return self.layers[0].k

    @property
    def n_out(self) -> int:
        return self.layers[-1].n

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
        return sum(2 * l.k_logical * l.n_logical for l in self.layers)

    @property
    def bytes_per_row(self) -> int:
        return 2 * (self.k0 + self.n_out)

    @property
    def weight_bytes(self) -> int:
        b = sum(2 * (l.k * l.n + l.n) for l in self.layers)
        if self.tail != L.TAIL_NONE:
            b += 4 * self.n_out
        return b

    def spec(self) -> L.GpSpec:
        return L.make_spec(self.widths, self.acts, self.tail, self.gp_dtype, self.ln_eps)

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

WORKLOADS = {w.name: w for w in (MGN_EDGE, MGN_NODE, MGN_LINEARS, TEST_MLP)}


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
        ln = (torch.ones(w.n_out, dtype=w.dtype), torch.zeros(w.n_out, dtype=w.dtype))
    return layers, ln


def make_input_chunk(w: Workload, chunk: int, rows: int | None = None) -> torch.Tensor:
    """Rows [chunk*CHUNK_ROWS, chunk*CHUNK_ROWS + rows) of the input, in w.dtype."""
    rows = CHUNK_ROWS if rows is None else rows
    g = _gen(w.seed, 1, chunk)
    if w.input_kind == "normal":
        x = torch.randn(rows, w.k0, generator=g)
    else:
        raise ValueError(w.input_kind)
    if w.input_logical < w.k0:
        x[:, w.input_logical:] = 0
    return x.to(w.dtype)


def make_input(w: Workload, row0: int = 0, rows: int | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows [row0, row0+rows) of the input (host tensor, optionally written into `out`)."""
    rows = w.m - row0 if rows is None else rows
    if out is None:
        out = torch.empty(rows, w.k0, dtype=w.dtype)
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
