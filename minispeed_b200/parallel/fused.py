"""Fused in-kernel NVLink collectives (one rank per GPU of one node)."""

from __future__ import annotations

import torch


def supported(device: torch.device):
    return False, "fused NVLink collectives not built yet"


class FusedCollectives:  # pragma: no cover - placeholder until the peer runtime lands
    name = "fused"

    def __init__(self, *a, **k):
        raise RuntimeError("fused collectives unavailable")
