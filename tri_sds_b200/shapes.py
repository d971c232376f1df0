"""Model-shape configuration (Qwen3 family) for the device path."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class QwenShape:
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    n_layers: int
    vocab: int
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6
    qk_norm: bool = True
    tie_embeddings: bool = False

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def q_per_kv(self) -> int:
        return self.n_heads // self.n_kv_heads

    def layer_params(self) -> int:
        N, I = self.hidden, self.intermediate
        return N * self.qkv_dim + self.q_dim * N + 3 * N * I + 2 * N + 2 * self.head_dim

    def layer_weight_bytes(self) -> int:
        """bf16 bytes of the four projections of one layer (what a forward streams)."""
        N, I = self.hidden, self.intermediate
        return 2 * (N * self.qkv_dim + self.q_dim * N + 3 * N * I)

    def lm_head_bytes(self) -> int:
        return 2 * self.vocab * self.hidden


# The two shapes of the workloads: a Qwen3-32B-shape target and a
# Qwen3-4B-shape draft (tied embeddings), both with QK-norm.
QWEN3_32B = QwenShape(5120, 64, 8, 128, 25600, 64, 151936)
QWEN3_4B = QwenShape(2560, 32, 8, 128, 9728, 36, 151936, tie_embeddings=True)
