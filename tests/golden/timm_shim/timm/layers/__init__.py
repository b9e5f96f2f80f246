"""timm.layers names the reference imports (own minimal versions)."""
import torch
import torch.nn as nn


class Mlp(nn.Module):
    """fc1 -> act -> fc2 (the parameterised layers carry timm's names)."""

    def __init__(self, in_features=None, hidden_features=None, out_features=None,
                 act_layer=nn.GELU, drop=0.0, bias=True, **_):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features, bias=bias)
        self.act = act_layer()
        self.drop1 = nn.Dropout(drop)
        self.norm = nn.Identity()
        self.fc2 = nn.Linear(hidden_features, out_features, bias=bias)
        self.drop2 = nn.Dropout(drop)

    def forward(self, x):
        return self.drop2(self.fc2(self.norm(self.drop1(self.act(self.fc1(x))))))


class DropPath(nn.Module):
    """Stochastic depth; the identity at inference, which is all the
    fixtures run."""

    def __init__(self, drop_prob=0.0, **_):
        super().__init__()
        self.drop_prob = drop_prob

    def forward(self, x):
        if not self.training or self.drop_prob == 0.0:
            return x
        keep = 1.0 - self.drop_prob
        mask = x.new_empty((x.shape[0],) + (1,) * (x.ndim - 1)).bernoulli_(keep)
        return x * mask / keep


def use_fused_attn(*_args, **_kwargs):
    return True


def trunc_normal_(tensor, mean=0.0, std=1.0, a=-2.0, b=2.0):
    return nn.init.trunc_normal_(tensor, mean=mean, std=std, a=a, b=b)


__all__ = ["Mlp", "DropPath", "use_fused_attn", "trunc_normal_", "torch"]
