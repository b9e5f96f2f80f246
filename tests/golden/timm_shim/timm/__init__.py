"""Minimal stand-in for the timm package, written for this repository and
used ONLY by the fixture generators under tests/golden (make_golden.py,
make_model_golden.py).

timm is not installed here.  The reference's modules import a handful of its
names; this package provides them as small PyTorch modules of its own with
the same constructor arguments, attribute names and forward semantics the
reference relies on (a pre-norm ViT: patch embedding, CLS token and position
embedding, blocks of attention + MLP with LayerNorm eps 1e-6, a final norm).
It is not timm's code; it is never imported by the product or by tests that
run on the GPU box.
"""
