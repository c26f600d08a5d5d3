"""The five encoder-policy workloads (configs C1-C5) as host-side configs.

Mirrors ow_policy_preset() of the C ABI field for field; a test checks the two
agree.
"""
from __future__ import annotations

from dataclasses import dataclass, replace, asdict

PRECISION = {"f32": 0, "bf16": 1, "fp8": 2}
DTYPE = {"f32": 0, "bf16": 1}
IO = {"host": 0, "device": 1}


@dataclass(frozen=True)
class PolicyConfig:
    name: str
    batch: int            # states per forward (batch_capacity)
    n_entities: int       # N
    features: int         # F
    d_model: int
    heads: int
    ffn: int
    layers: int
    actions: int          # P
    count_lo: int
    count_hi: int
    precision: str        # f32 | bf16 | fp8
    sample_actions: bool
    logits_dtype: str     # f32 | bf16
    value_dtype: str      # f32 | bf16
    onehot_features: bool = False  # C4: channels 16..31 are four one-hot blocks of 4

    def with_(self, **kw) -> "PolicyConfig":
        return replace(self, **kw)

    def as_dict(self) -> dict:
        return asdict(self)

    def flops_per_state(self) -> float:
        """Dense padded forward FLOPs per state: 2NFd + L(8Nd^2 + 4Ndf + 4N^2 d) + 2NdP + 2d."""
        N, F, d, f, L, P = self.n_entities, self.features, self.d_model, self.ffn, self.layers, self.actions
        return 2 * N * F * d + L * (6 * N * d * d + 2 * N * d * d + 4 * N * d * f + 4 * N * N * d) + 2 * N * d * P + 2 * d

    def gemm_flops_per_token(self) -> float:
        """Block-GEMM FLOPs per valid token (QKV + out-proj + FFN up + FFN down) over all layers."""
        d, f = self.d_model, self.ffn
        return self.layers * (2 * d * 3 * d + 2 * d * d + 2 * d * f + 2 * f * d)


PRESETS = {
    1: PolicyConfig("C1-tiny-fp32", 64, 32, 16, 128, 4, 512, 2, 8, 8, 32, "f32", False, "f32", "f32"),
    2: PolicyConfig("C2-medium-bf16", 1024, 64, 32, 256, 8, 1024, 4, 16, 16, 64, "bf16", False, "bf16", "f32"),
    3: PolicyConfig("C3-medium-fp8", 4096, 64, 32, 256, 8, 1024, 4, 16, 16, 64, "fp8", False, "bf16", "bf16"),
    4: PolicyConfig("C4-rollout-bf16-gumbel", 8192, 96, 32, 384, 12, 1536, 6, 16, 24, 96, "bf16", True, "bf16", "f32",
                    onehot_features=True),
    5: PolicyConfig("C5-large-bf16", 65536, 128, 32, 512, 16, 2048, 8, 16, 32, 128, "bf16", False, "bf16", "f32"),
}


def preset(i: int) -> PolicyConfig:
    return PRESETS[int(i)]
