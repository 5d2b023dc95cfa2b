"""comfy_kitchen's rms_rope_split_half_ restated with the oracle's convention (in place)."""
import numpy as np
import torch

from oracle import h3_oracle as O


class _CK:
    @staticmethod
    def rms_rope_split_half_(q, k, rope_freqs, qw, kw, epsilon=1e-6, rot_dim=128):
        # q, k: [1, S, H, 128] views into the fused QKV output; rope_freqs: [1, S, 64, 2, 2]
        assert rot_dim == 128
        rope = rope_freqs[0].detach().float().cpu().numpy()
        for t, w in ((q, qw), (k, kw)):
            x = t[0].detach().float().cpu().numpy()
            wn = None if w is None else O.bf16_round(w.detach().float().cpu().numpy())
            y = O.qknorm_rope(O.bf16_round(x), wn, rope, float(epsilon))
            t[0].copy_(torch.from_numpy(y).to(t.dtype))


ck = _CK()
