"""Test-only stand-in for the parts of ComfyUI that harness/sp_runtime.py imports, so the
reference runtime (and this repo's drop-in) can run on CPU gloo ranks."""
