"""B200-native (sm_100a) DiT-block hot path of the MiniMax-H3 video DiT.

Drop-in surface (mirrors BHUHD/minixmax-h3 h3_npu): ``QuantLinear`` /
``Ops`` (modules/linear.py), ``h3_attention_bnsd`` (ops/fa_h3.py), Ulysses
``all_to_all_heads`` / ``split_range`` / ``clip_mod_segments``
(ops/ulysses.py) and ``DiTBlock`` (model/dit.py).  Compute runs in the
hand-written CUDA kernels of ``libh3b.so`` (C ABI: include/h3b.h).
"""
from __future__ import annotations

__version__ = "0.1.0"
