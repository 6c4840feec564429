"""Shape of the Laya decision network served by the b200 mode.

The reference never hard-codes these numbers in one place: the encoder comes
from the checkpoint's ``encoder/config.json`` (ModernBERT-large shaped, 28
layers, d=1024, 16 heads of 64, intermediate 2624, vocab 50368, global
attention every third layer with RoPE theta 160000, radius-64 local windows
with theta 10000) and the head from the Laya SDK (two pre-norm
``nn.TransformerEncoderLayer`` with 16 heads and a 4096 ReLU FFN, a
``type_emb`` table, ``scorer`` and ``act_head``).  The reference reads them at
``src/laya_blackwell/model.py:37-56`` (heads, head dim, max positions, global
layer flags, RoPE tables) and ``model.py:82-83`` (window = local_attention//2).
"""
from dataclasses import dataclass, asdict, field


@dataclass(frozen=True)
class LayaConfig:
    layers: int = 28
    hidden: int = 1024
    heads: int = 16
    head_dim: int = 64
    intermediate: int = 2624
    vocab: int = 50368
    pad_token_id: int = 50283
    max_len: int = 512
    local_attention: int = 128          # total window; radius = local_attention // 2
    global_every: int = 3               # layer i is global iff i % global_every == 0
    rope_theta_global: float = 160000.0
    rope_theta_local: float = 10000.0
    norm_eps: float = 1e-5
    head_layers: int = 2
    head_heads: int = 16
    head_ff: int = 4096
    num_qtypes: int = 3
    act_hidden: int = 256
    act_features: int = 4               # top1, top1-top2, entropy, count/255 (model.py:120)

    @property
    def window(self):
        return self.local_attention // 2

    def is_global(self, layer):
        return layer % self.global_every == 0

    def as_dict(self):
        return asdict(self)

    def validate(self):
        if self.head_dim != 64:
            raise ValueError("the b200 kernels are built for a head dimension of 64")
        if self.hidden != self.heads * self.head_dim:
            raise ValueError("hidden must equal heads * head_dim")
        if self.hidden % 128 or self.hidden > 4096:
            raise ValueError("hidden must be a multiple of 128 and at most 4096")
        if self.intermediate % 64:
            raise ValueError("intermediate must be a multiple of 64")
        if self.head_ff % 128:
            raise ValueError("head_ff must be a multiple of 128")
        if not 1 <= self.max_len <= 512:
            raise ValueError("max_len must be in [1, 512]: attention keeps a query's scores in tensor memory")
        if self.hidden // self.head_heads != 64:
            raise ValueError("head attention must also use 64-wide heads")
        if self.act_hidden % 32 or self.act_hidden > 1024:
            raise ValueError("act_hidden must be a multiple of 32 and at most 1024")
        return self


LAYA = LayaConfig()

# Small network with the same structure, for fast CPU checks and kernel tests.
TINY = LayaConfig(layers=4, hidden=256, heads=4, intermediate=384, vocab=1000,
                  pad_token_id=999, max_len=512, head_heads=4, head_ff=512,
                  act_hidden=64)
