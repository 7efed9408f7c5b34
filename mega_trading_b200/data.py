"""Synthetic composite order-flow token streams, generated on the device.

The reference tokenises Binance trades into one mixed-radix id per event
(``src/mega_trading/tokenizer.py:121-143, :270-274``) and trains on
``input_ids = t[:-1], labels = t[1:]`` windows (``dataset.py:134-140``).  The
archives are not available offline, so training and benchmarks draw the token
fields independently per seed (the BASELINE stand-in):

  action, side ~ U{0, 1};  depth = min(Geometric(p=0.3) - 1, 20);
  volume, interarrival = min(Zipf(s=1.2) - 1, 15);
  id = (((action * 2 + side) * 21 + depth) * 16 + volume) * 16 + interarrival

giving a vocabulary of 2 * 2 * 21 * 16 * 16 = 21,504 ids.
"""

from __future__ import annotations

import math

import torch

VOCAB_SIZE = 2 * 2 * 21 * 16 * 16


def _zipf_clipped_probs(s: float = 1.2, cap: int = 15) -> torch.Tensor:
    """P(min(Z - 1, cap) = k) for Z ~ Zipf(s): k^-s / zeta(s) for k < cap, tail mass at cap."""
    # zeta(s) by direct summation plus the Euler-Maclaurin tail estimate
    n = 10_000
    head = sum(k ** -s for k in range(1, n))
    tail = n ** (1 - s) / (s - 1) + 0.5 * n ** -s + s * n ** (-s - 1) / 12
    zeta = head + tail
    probs = [(k + 1) ** -s / zeta for k in range(cap)]
    probs.append(1.0 - sum(probs))
    return torch.tensor(probs, dtype=torch.float64)


_ZIPF = _zipf_clipped_probs()


def composite_tokens(batch: int, length: int, *, seed: int, device: torch.device | str = "cpu") -> torch.Tensor:
    """``[batch, length]`` int64 composite-token ids drawn from the BASELINE distribution."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    shape = (batch, length)
    action = torch.randint(0, 2, shape, generator=g, device=device)
    side = torch.randint(0, 2, shape, generator=g, device=device)
    depth = torch.empty(shape, device=device, dtype=torch.float32).geometric_(0.3, generator=g).long() - 1
    depth = depth.clamp_(max=20)
    zipf = _ZIPF.to(device=device, dtype=torch.float32)
    vol = torch.multinomial(zipf, batch * length, replacement=True, generator=g).view(shape)
    dt = torch.multinomial(zipf, batch * length, replacement=True, generator=g).view(shape)
    return (((action * 2 + side) * 21 + depth) * 16 + vol) * 16 + dt


def next_token_batch(batch: int, seq_len: int, *, seed: int, device: torch.device | str = "cpu"):
    """``(input_ids, labels)`` of shape ``[batch, seq_len]`` from one window of ``seq_len + 1`` tokens."""
    t = composite_tokens(batch, seq_len + 1, seed=seed, device=device)
    return t[:, :-1], t[:, 1:]


assert VOCAB_SIZE == 21504 and math.isclose(float(_ZIPF.sum()), 1.0, rel_tol=1e-9)
