"""Inert placeholders: the routing path never builds these."""
import torch.nn as nn


class LayerScale(nn.Module):
    def __init__(self, dim, init_values=1e-5, inplace=False):
        super().__init__()
        self.gamma = nn.Parameter(init_values * __import__("torch").ones(dim))

    def forward(self, x):
        return x * self.gamma


class Attention(nn.Module):
    pass


class Block(nn.Module):
    pass


class VisionTransformer(nn.Module):
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("placeholder: the real timm is not installed")
