"""Channel helpers named as the reference imports them (chunk.py:44)."""

import torch


class dotdict(dict):
    """dict with attribute access (the reference reads ``config.x`` and ``config.get``)."""

    __getattr__ = dict.get
    __setattr__ = dict.__setitem__
    __delattr__ = dict.__delitem__

    def __deepcopy__(self, memo):
        import copy
        return dotdict(copy.deepcopy(dict(self), memo))


def interleave(z_pre: torch.Tensor) -> torch.Tensor:
    """[B, 3H, T]: channel 3h+j -> group j (concatenated groups 0, 1, 2)."""
    return torch.cat([z_pre[:, 0::3], z_pre[:, 1::3], z_pre[:, 2::3]], dim=1)


def column_split(z_pre, num_heads, head_size):
    raise NotImplementedError("column_split_hyena is not used by the restated model")
