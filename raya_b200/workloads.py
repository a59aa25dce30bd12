"""The benchmark workloads (synthetic inputs; the reference has no dataset).

Five configurations of block-local attention, all fp32 and head_dim 64:

  c1  batch 1,  12 heads, seq 512,  block 64,  seed 0, N(0,1), no padding
  c2  batch 32, 12 heads, seq 1024, block 64,  seed 1, N(0,1), valid ~ U[512, 1024]
  c3  batch 16, 12 heads, seq 2048, block {32, 64, 128, 256}, seed 2, N(0,1), no padding
  c4  12 layers x (batch 64, 12 heads, seq 512, block 64), seed 3+layer, N(0, 0.5^2),
      valid ~ U[128, 512] (the same batch of sequences through every layer)
  c5  batch 256, 16 heads, seq 8192, block 128, seed 4, N(0,1), valid ~ U[4096, 8192]

The mask is block-local with a halo: halo 1 is raya's Block3 (query block b
sees key blocks b-1..b+1), halo 0 is "own block only".

Values: element i of tensor t (q = 0, k = 1, v = 2) of a configuration is a
function of (seed, t, i) only (``raya_attn_fill_normal``: splitmix64 ->
Box-Muller), so a shard of the batch is generated on its own GPU without any
data movement.  Valid lengths: ``valid_lengths`` (splitmix64, uniform
integers in [lo, hi]).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

MASK64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    """splitmix64 (Steele, Lea, Flood 2014), the generator's mixing step."""
    x = (x + 0x9E3779B97F4A7C15) & MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK64
    return x ^ (x >> 31)


def valid_lengths(seed: int, batch: int, lo: int, hi: int, first: int = 0) -> np.ndarray:
    """Uniform integers in [lo, hi] for batch entries first .. first+batch-1."""
    span = hi - lo + 1
    key = splitmix64((seed * 0x9E3779B97F4A7C15 + 0x5EED) & MASK64)
    return np.array([lo + splitmix64((key + first + b) & MASK64) % span for b in range(batch)],
                    dtype=np.int32)


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    heads: int
    seq: int
    head_dim: int
    block: int
    halo: int
    seed: int
    stddev: float
    valid: tuple[int, int] | None  # (lo, hi) or None = no padding
    layers: int = 1

    def valid_len(self, first: int = 0, count: int | None = None) -> np.ndarray:
        n = self.batch if count is None else count
        if self.valid is None:
            return np.full(n, self.seq, dtype=np.int32)
        return valid_lengths(self.seed, n, self.valid[0], self.valid[1], first)

    def layer_seed(self, layer: int) -> int:
        return self.seed + layer

    @property
    def numel(self) -> int:
        return self.batch * self.heads * self.seq * self.head_dim

    def with_halo(self, halo: int) -> "Workload":
        return replace(self, halo=halo)


CONFIGS: dict[str, Workload] = {
    "c1": Workload("c1", 1, 12, 512, 64, 64, 1, 0, 1.0, None),
    "c2": Workload("c2", 32, 12, 1024, 64, 64, 1, 1, 1.0, (512, 1024)),
    "c3-b32": Workload("c3-b32", 16, 12, 2048, 64, 32, 1, 2, 1.0, None),
    "c3-b64": Workload("c3-b64", 16, 12, 2048, 64, 64, 1, 2, 1.0, None),
    "c3-b128": Workload("c3-b128", 16, 12, 2048, 64, 128, 1, 2, 1.0, None),
    "c3-b256": Workload("c3-b256", 16, 12, 2048, 64, 256, 1, 2, 1.0, None),
    "c4": Workload("c4", 64, 12, 512, 64, 64, 1, 3, 0.5, (128, 512), layers=12),
    "c5": Workload("c5", 256, 16, 8192, 64, 128, 1, 4, 1.0, (4096, 8192)),
    # c5's sequences at 1/32 of its batch (about 1 GB on the device): the
    # size at which ncu captures the c5 kernel (its traffic scales by
    # algorithmic bytes to the full c5 launch); not a benchmark line.
    "c5-p": Workload("c5-p", 8, 16, 8192, 64, 128, 1, 4, 1.0, (4096, 8192)),
}


def fill_device(w: Workload, tensors, layer: int = 0, bh0: int = 0, stream=None) -> None:
    """Fills device tensors (q, k, v) holding flattened slices [bh0, ...)
    of workload ``w`` (layer ``layer``)."""
    from .attention import fill_normal

    first = bh0 * w.seq * w.head_dim
    for t, x in enumerate(tensors):
        fill_normal(x, w.layer_seed(layer), t, first, w.stddev, stream)
