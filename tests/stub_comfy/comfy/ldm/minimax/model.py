"""ComfyUI-shaped H3 model module for tests: re-exports the repo's host-model stand-in."""
from h3_model import (AdalnProj, Attention, DiTBlock, MiniMaxH3Model, MLP, RMSNorm,  # noqa: F401
                      _mod_gate, _mod_scale_shift, init_weights, rope_freqs_1d, timestep_embedding)
