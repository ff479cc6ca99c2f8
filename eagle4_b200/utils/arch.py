"""Hardware check: this package's kernels are built for sm_100a (B200 / GB200) only.

``require_sm100(device)`` raises with the device's name and compute capability on anything else, so an unsupported
GPU is refused at load time with a reason instead of failing inside a kernel (reference hardware dispatch:
``eagle_harness/kernels/arch.py``, which also routes AMD GPUs to other kernels; this package has one target).
"""

from __future__ import annotations

from typing import Optional

import torch

SUPPORTED = {(10, 0)}  # sm_100 (B200, GB200): tcgen05 / TMEM / TMA kernels built for sm_100a


class UnsupportedDevice(RuntimeError):
    pass


def capability(device: Optional[torch.device] = None):
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return torch.cuda.get_device_capability(dev), torch.cuda.get_device_name(dev)


def require_sm100(device: Optional[torch.device] = None) -> None:
    if not torch.cuda.is_available():
        raise UnsupportedDevice("no CUDA device: the sm_100a kernels need a B200-class GPU")
    cap, name = capability(device)
    if tuple(cap) not in SUPPORTED:
        raise UnsupportedDevice(f"{name} (sm_{cap[0]}{cap[1]}) is not supported: eagle4_b200 kernels are built for "
                                "sm_100a (B200 / GB200) only")
