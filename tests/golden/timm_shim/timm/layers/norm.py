from torch.nn import LayerNorm  # noqa: F401
