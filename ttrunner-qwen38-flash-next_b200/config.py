"""Shapes of the qwen4exp MoE block and how a rank's shard is described.

`MoEConfig` carries the MoE fields of the reference's Qwen4ExpConfig
(reference/config.py:44-48: num_experts, num_experts_per_tok,
expert_intermediate, shared_expert_intermediate) plus the hidden size and
layer count.  `Shard` names the two expert partitions the reference plans
(tt/plan.py:31-49, 70-103): variant "A" splits the expert axis (rank r holds
experts [r*E/n, (r+1)*E/n), the shared expert lives on rank 0), variant "B"
splits every expert's intermediate axis (rank r holds gate/up rows and down
columns [r*I/n, (r+1)*I/n), the shared expert split the same way).
"""

from __future__ import annotations

from dataclasses import dataclass

from ._lib import Dims

SB_VALUES = 256
SB_BYTES = 136


def iq4xs_bytes(n_values: int) -> int:
    if n_values % SB_VALUES:
        raise ValueError(f"{n_values} values is not a whole number of IQ4_XS super-blocks")
    return n_values // SB_VALUES * SB_BYTES


@dataclass(frozen=True)
class MoEConfig:
    hidden: int = 2048
    inter: int = 512
    n_experts: int = 512
    top_k: int = 10
    shared_inter: int = 512
    n_layers: int = 1
    weight_std: float = 0.02
    # std of the down projections (routed and shared); None: weight_std.  Tests use a larger one
    # so that a literal stack keeps its activations near unit RMS through every layer.
    down_std: float | None = None

    @property
    def dn_std(self) -> float:
        return self.weight_std if self.down_std is None else self.down_std

    @property
    def gate_up_row_bytes(self) -> int:
        return iq4xs_bytes(self.hidden)

    @property
    def down_row_bytes(self) -> int:
        return iq4xs_bytes(self.inter)

    @property
    def expert_bytes(self) -> int:
        """IQ4_XS bytes of one routed expert (gate|up + down)."""
        return 2 * self.inter * self.gate_up_row_bytes + self.hidden * self.down_row_bytes

    @property
    def shared_bytes(self) -> int:
        return 2 * self.shared_inter * self.gate_up_row_bytes + self.hidden * iq4xs_bytes(self.shared_inter)

    @property
    def router_bytes(self) -> int:
        return self.n_experts * self.hidden * 4

    def layer_expert_bytes(self, n_unique: int | None = None) -> int:
        """Algorithmic bytes of one layer: the routed experts read plus the shared one."""
        n = self.top_k if n_unique is None else n_unique
        return n * self.expert_bytes + self.shared_bytes


# BASELINE configurations (shapes only; seeds live with the generators).
C1 = MoEConfig(n_layers=1)
C2 = MoEConfig(n_layers=48)


@dataclass(frozen=True)
class Shard:
    variant: str = "none"   # "none", "A" (expert axis) or "B" (intermediate axis)
    rank: int = 0
    world: int = 1

    def __post_init__(self) -> None:
        if self.variant not in ("none", "A", "B"):
            raise ValueError(f"unknown shard variant {self.variant!r}")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world {self.world}")
        if self.variant == "none" and self.world != 1:
            raise ValueError("variant 'none' is a single rank")

    def expert_window(self, cfg: MoEConfig) -> tuple[int, int]:
        if self.variant != "A":
            return 0, cfg.n_experts
        if cfg.n_experts % self.world:
            raise ValueError(f"{cfg.n_experts} experts do not split over {self.world} ranks")
        per = cfg.n_experts // self.world
        return self.rank * per, (self.rank + 1) * per

    def inter_window(self, inter: int) -> tuple[int, int]:
        if self.variant != "B":
            return 0, inter
        if inter % (32 * self.world):
            raise ValueError(f"intermediate {inter} does not split into 32-value blocks over {self.world}")
        per = inter // self.world
        return self.rank * per, (self.rank + 1) * per

    def has_shared(self) -> bool:
        return self.variant != "A" or self.rank == 0

    @staticmethod
    def row_slice(lo: int, hi: int) -> tuple[int, int, int]:
        """(segments, sub-blocks per segment, first sub-block) for columns [lo, hi) of an IQ4_XS row."""
        width = hi - lo
        if lo % 256 == 0 and width % 256 == 0:
            return width // 256, 8, 0
        if lo // 256 != (hi - 1) // 256 or lo % 32 or width % 32:
            raise ValueError(f"column slice [{lo}, {hi}) crosses a super-block unevenly")
        return 1, width // 32, (lo % 256) // 32

    def dims(self, cfg: MoEConfig) -> Dims:
        e_lo, e_hi = self.expert_window(cfg)
        i_lo, i_hi = self.inter_window(cfg.inter)
        nseg, nsub, ib0 = self.row_slice(i_lo, i_hi)
        d = Dims(
            hidden=cfg.hidden, inter=cfg.inter, n_experts=cfg.n_experts, top_k=cfg.top_k,
            expert_lo=e_lo, expert_hi=e_hi, inter_local=i_hi - i_lo,
            down_nseg=nseg, down_nsub=nsub, down_ib0=ib0,
        )
        if self.has_shared() and cfg.shared_inter > 0:
            s_lo, s_hi = self.inter_window(cfg.shared_inter)
            snseg, snsub, sib0 = self.row_slice(s_lo, s_hi)
            d.sh_inter_local = s_hi - s_lo
            d.sh_down_nseg, d.sh_down_nsub, d.sh_down_ib0 = snseg, snsub, sib0
        return d
