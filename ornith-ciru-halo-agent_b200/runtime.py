"""One shared workspace arena and per-layer sticky error flags.

Mirrors plugin-site/ornith_g256/runtime.py:13-97 for the routed path: one
workspace sized for `capacity` rows serves every layer (calls are serialised
on one stream), each layer owns one uint32 flag slot that the library ORs
into, flags are reset only outside CUDA-graph capture, and a check raises on
any non-zero slot.  Bit 4 (invalid expert id) is fatal; bits 1/2/8/16/32 are
numerical (worker.py:189-197, mask 59); bit 64 means a bounded device wait
gave up, and bit 128 (debug-bounds builds only) that an index outside its
buffer was redirected.
"""
import torch

from . import native

NUMERIC_MASK = 59


class Runtime:
    """`layers` names the layers that own a flag slot (in slot order);
    `dense_shapes` lists the (N, K) of the dense G256 layers sharing the arena
    and `head` says whether the W8 head does (runtime.py:36-40 sizes the arena
    the same way).  Settings: the routed activation bits of native.configure,
    dense_geometry / head_geometry (0, 1 or 2) and dense_a8_max_rows (32 or
    64, the row count up to which dense calls take the A8 projection)."""

    def __init__(self, layers, capacity, device, settings=None, dense_shapes=(), head=False):
        settings = settings or {}
        self.capacity = int(capacity)
        self.device = torch.device(device)
        self.dense_geometry = settings.get('dense_geometry', 2)
        self.dense_a8_max_rows = settings.get('dense_a8_max_rows', 32)
        if self.dense_a8_max_rows not in (32, 64):
            raise ValueError(f'dense_a8_max_rows is {self.dense_a8_max_rows}; it must be 32 or 64')
        self.head_geometry = settings.get('head_geometry', 2)
        if self.dense_geometry not in (0, 1, 2) or self.head_geometry not in (0, 1, 2):
            raise ValueError('dense_geometry and head_geometry take 0, 1 or 2')
        size = native.configure(settings, self.capacity)
        if dense_shapes:
            size = max(size, native.dense_workspace_bytes(self.capacity, sorted(set(dense_shapes))))
        if head:
            size = max(size, native.head_get_layout(native.HEAD_ROWS).workspace_bytes)
        self.workspace = torch.empty(size, dtype=torch.uint8, device=self.device)
        self.error_flags = torch.zeros(len(layers), dtype=torch.int32, device=self.device)
        self.slots = tuple(self.error_flags[i:i + 1] for i in range(len(layers)))
        self.layer_prefixes = tuple(layers)

    def reset_error_flags(self):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError('error flags are reset outside CUDA graph capture only')
        self.error_flags.zero_()

    def check_error_flags(self):
        flags = self.error_flags.cpu().tolist()
        if any(flags):
            raise RuntimeError(f'native error flags set: '
                               f'{ {name: code for name, code in zip(self.layer_prefixes, flags) if code} }')
        return flags
