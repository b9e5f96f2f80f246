"""Inert placeholders for the timm.layers names the reference imports."""
import torch.nn as nn


class Mlp(nn.Module):
    def __init__(self, in_features=None, hidden_features=None, out_features=None,
                 act_layer=nn.GELU, drop=0.0, **_):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features)
        self.act = act_layer()
        self.fc2 = nn.Linear(hidden_features, out_features)

    def forward(self, x):
        return self.fc2(self.act(self.fc1(x)))


class DropPath(nn.Identity):
    def __init__(self, *args, **kwargs):
        super().__init__()


def use_fused_attn(*_args, **_kwargs):
    return True


def trunc_normal_(tensor, mean=0.0, std=1.0, a=-2.0, b=2.0):
    return nn.init.trunc_normal_(tensor, mean=mean, std=std, a=a, b=b)
