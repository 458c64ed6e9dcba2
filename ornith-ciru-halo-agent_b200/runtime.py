"""One shared workspace arena and per-layer sticky error flags.

Mirrors plugin-site/ornith_g256/runtime.py:13-97 for the routed path: one
workspace sized for `capacity` rows serves every layer (calls are serialised
on one stream), each layer owns one uint32 flag slot that the library ORs
into, flags are reset only outside CUDA-graph capture, and a check raises on
any non-zero slot.  Bit 4 (invalid expert id) is fatal; bits 1/2/8/16/32 are
numerical (worker.py:189-197, mask 59); bit 64 means a bounded device wait
gave up.
"""
import torch

from . import native

NUMERIC_MASK = 59


class Runtime:
    def __init__(self, layers, capacity, device, settings=None):
        self.capacity = int(capacity)
        self.device = torch.device(device)
        size = native.configure(settings or {}, self.capacity)
        self.workspace = torch.empty(size, dtype=torch.uint8, device=self.device)
        self.error_flags = torch.zeros(len(layers), dtype=torch.int32, device=self.device)
        self.slots = tuple(self.error_flags[i:i + 1] for i in range(len(layers)))
        self.layer_prefixes = tuple(layers)

    def reset_error_flags(self):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError('Reset native error flags outside graph capture')
        self.error_flags.zero_()

    def check_error_flags(self):
        flags = self.error_flags.cpu().tolist()
        if any(flags):
            raise RuntimeError(str({name: code for name, code in zip(self.layer_prefixes, flags) if code}))
        return flags
