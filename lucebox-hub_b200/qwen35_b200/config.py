"""Model dimensions of the Qwen3.5 hybrid (Gated-DeltaNet + gated full-attention) forward path.

The 0.8B numbers restate the constants of the reference package
(models/qwen35_0p8b/model.py:7-42, models/qwen35_0p8b/kernel.cu:23-49); the CUDA
kernels are compiled for exactly these.  `Dims` is also instantiated at tiny sizes
by the CPU oracle tests.
"""
from dataclasses import dataclass, field
from typing import List


@dataclass(frozen=True)
class Dims:
    num_layers: int = 24
    hidden: int = 1024
    intermediate: int = 3584
    vocab: int = 248320
    # gated full attention
    fa_q_heads: int = 8
    fa_kv_heads: int = 2
    fa_head_dim: int = 256
    fa_rotary_dim: int = 64
    rope_theta: float = 1.0e7
    # gated DeltaNet
    dn_heads: int = 16          # value heads
    dn_k_heads: int = 16        # key heads (27B: 16 key heads shared by 48 value heads)
    dn_key_dim: int = 128
    dn_value_dim: int = 128
    dn_conv_kernel: int = 4
    rms_eps: float = 1e-6
    full_attention_interval: int = 4

    @property
    def layer_types(self) -> List[int]:
        """0 = DeltaNet, 1 = full attention (models/qwen35_0p8b/model.py:37)."""
        return [1 if (i + 1) % self.full_attention_interval == 0 else 0
                for i in range(self.num_layers)]

    @property
    def n_fa(self) -> int:
        return sum(self.layer_types)

    @property
    def n_dn(self) -> int:
        return self.num_layers - self.n_fa

    @property
    def fa_q_size(self) -> int:
        return self.fa_q_heads * self.fa_head_dim

    @property
    def fa_qproj_size(self) -> int:
        return 2 * self.fa_q_size

    @property
    def fa_kv_size(self) -> int:
        return self.fa_kv_heads * self.fa_head_dim

    @property
    def dn_qk_size(self) -> int:
        return self.dn_k_heads * self.dn_key_dim

    @property
    def dn_v_size(self) -> int:
        return self.dn_heads * self.dn_value_dim

    @property
    def dn_conv_channels(self) -> int:
        return 2 * self.dn_qk_size + self.dn_v_size


QWEN35_0P8B = Dims()

# A small instance with the same structure (two [DN,DN,DN,FA] groups) for CPU tests.
TINY = Dims(num_layers=8, hidden=64, intermediate=160, vocab=512,
            fa_q_heads=4, fa_kv_heads=2, fa_head_dim=32, fa_rotary_dim=8,
            dn_heads=4, dn_k_heads=4, dn_key_dim=16, dn_value_dim=16)

MAX_SEQ_LEN = 2048  # default cache length of the reference Decoder (model.py:11)
