"""Packed-weight methods the reference plugin drives: routed experts, dense
G256 linears and the W8 head.

Mirrors, without vLLM, the reference plugin's methods and its strict
checkpoint loaders:
  * `register_packed`, `G256LinearMethod`, `W8HeadMethod`
    (plugin-site/ornith_g256/method.py:11-91): packed parameters that accept
    one load each of their exact shape and dtype, sealed after loading, and
    `apply` through `ornith_b200::dense_out` / `ornith_b200::head_out`;
  * `G256MoEMethod` (plugin-site/ornith_g256/method.py:101-184):
    `create_weights` registers the four N16 tile banks of a routed layer,
    `process_weights_after_loading` seals them, `prepare_n32_weights` reorders
    them once into the N32 storage this library computes on, and `apply(layer,
    x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None)`
    returns a fresh bf16 output through `ornith_b200::routed_out`;
  * `install_tilebank_loader` / `require_complete_tilebank_load`
    (plugin-site/ornith_g256/loader.py:12-54): a checkpoint stream of
    `routed_experts.<field>` tensors is admitted only if every field is known,
    loaded once, of the registered shape and dtype, materialised, and (for the
    metadata) CPU uint32 fp16 pairs with finite offsets and scales at or above
    the 2^-14 floor.  The kernels trust the banks, so these checks are the
    only guard against a malformed checkpoint.
The layer is any torch.nn.Module (vLLM's FusedMoE in the reference).  The
N32 reorder runs on the GPU through `ornith_moe_b200_repack_n16_to_n32`.
"""
from types import MethodType

import torch

from . import native

FIELDS = ('w13_tilebank_codes', 'w13_tilebank_metadata', 'w2_tilebank_codes', 'w2_tilebank_metadata')
PREFIX = 'routed_experts.'
E, H, I = 256, 2048, 512
# (projection, N, K) of the two banks (method.py:117)
PROJECTIONS = (('w13', 2 * I, H), ('w2', H, I))


def _load_direct(self, weights):
    """Strict direct load of `routed_experts.<field>` tensors (loader.py:17-43).
    A generator, as vLLM's `load_weights` is: it yields each admitted name."""
    if getattr(self, '_ornith_weights_ready', False):
        raise ValueError('Tilebank weights already sealed')
    for key, value in weights:
        if not key.startswith(PREFIX) or key[len(PREFIX):] not in FIELDS:
            raise ValueError('Unsupported tilebank checkpoint field ' + key)
        field = key[len(PREFIX):]
        if field in self._tilebank_loaded_fields:
            raise ValueError('Duplicate tilebank field ' + field)
        parameter = self._parameters.get(field)
        if parameter is None:
            raise ValueError('Missing registered tilebank parameter ' + field)
        if value.shape != parameter.shape or value.dtype != parameter.dtype:
            raise ValueError('Tilebank shape/dtype mismatch for ' + field)
        if value.device.type == 'meta' or parameter.device.type == 'meta':
            raise ValueError('Tilebank loader requires materialized tensors')
        if field.endswith('_metadata'):
            if value.device.type != 'cpu' or value.dtype != torch.uint32:
                raise ValueError('Tilebank metadata admission expects CPU uint32 packed pairs')
            # each word: fp16 scale (low half) | fp16 offset (high half)
            pairs = value.contiguous().view(torch.float16).reshape(*value.shape, 2)
            if not bool(torch.isfinite(pairs).all()) or not bool((pairs[..., 0] >= 2 ** -14).all()):
                raise ValueError('Tilebank metadata requires finite offset and normal-floor scale')
        with torch.no_grad():
            parameter.copy_(value)
        self._tilebank_loaded_fields.add(field)
        yield PREFIX + field


def install_tilebank_loader(layer):
    """Call once from create_weights, after the four bank parameters exist (loader.py:46-51)."""
    if hasattr(layer, '_tilebank_loaded_fields'):
        raise ValueError('Tilebank loader already installed')
    if any(name not in layer._parameters for name in FIELDS):
        raise ValueError('Create all four tilebank parameters first')
    layer._tilebank_loaded_fields = set()
    layer.load_weights = MethodType(_load_direct, layer)


def require_complete_tilebank_load(layer):
    """Call from process_weights_after_loading, before binding (loader.py:52-54)."""
    if getattr(layer, '_tilebank_loaded_fields', set()) != set(FIELDS):
        raise ValueError('Incomplete tilebank packed-bank checkpoint coverage')


def register_packed(layer, specs):
    """Register packed parameters (name, shape, dtype) whose weight_loader
    accepts one copy each of exactly that shape and dtype, before the layer
    is sealed (method.py:11-27)."""
    layer._g256_loaded = set()
    layer._g256_ready = False
    for name, shape, dtype in specs:
        param = torch.nn.Parameter(torch.empty(shape, dtype=dtype, device=getattr(layer, '_g256_device', None)),
                                   requires_grad=False)
        layer.register_parameter(name, param)

        def load(destination, value, *shard_args, name=name, param=param):
            if layer._g256_ready or name in layer._g256_loaded or destination is not param:
                raise ValueError(f'Duplicate or late packed load: {name}')
            if value.shape != param.shape or value.dtype != param.dtype:
                raise ValueError(f'Packed shape/dtype mismatch: {name}: {value.shape}/{value.dtype}')
            with torch.no_grad():
                param.copy_(value)
            layer._g256_loaded.add(name)
        param.weight_loader = load


class G256LinearMethod:
    """A dense G256 linear (method.py:30-62): codes uint32 [N/16, K/256, 32, 16]
    and metadata uint32 [N/16, K/256, 16]; apply(x [..., K]) -> bf16 [..., N]."""
    fields = ('g256_codes', 'g256_metadata')

    def __init__(self, prefix=''):
        self.prefix, self.runtime, self.slot = prefix, None, None

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **attrs):
        self.k, self.n = input_size, output_size
        if (input_size_per_partition != input_size or sum(output_partition_sizes) != output_size
                or getattr(layer, 'tp_size', 1) != 1 or params_dtype != torch.bfloat16
                or getattr(layer, 'has_bias', False) or not 0 < self.n <= 12288
                or self.n % 16 or not 0 < self.k <= 8192 or self.k % 256):
            raise ValueError(f'Unsupported G256 linear geometry: {self.prefix}: N{self.n}/K{self.k}')
        layer._g256_device = attrs.get('device')
        register_packed(layer, [(self.fields[0], (self.n // 16, self.k // 256, 32, 16), torch.uint32),
                                (self.fields[1], (self.n // 16, self.k // 256, 16), torch.uint32)])

    def process_weights_after_loading(self, layer):
        if layer._g256_loaded != set(self.fields):
            raise ValueError(f'Incomplete packed weights: {self.prefix}')
        layer._g256_ready = True

    def bind(self, runtime, slot):
        self.runtime, self.slot = runtime, slot

    def apply(self, layer, x, bias=None):
        if self.runtime is None or not layer._g256_ready or bias is not None:
            raise RuntimeError('G256 requires loaded weights and a bound worker')
        shape = x.shape[:-1]
        x = x.reshape(-1, self.k).contiguous()
        out = torch.empty((x.shape[0], self.n), dtype=x.dtype, device=x.device)
        native.dense_out(x, layer.g256_codes, layer.g256_metadata, self.runtime.workspace, out,
                         self.runtime.slots[self.slot], self.runtime.capacity, self.n, self.k,
                         self.runtime.dense_geometry, self.runtime.dense_a8_max_rows)
        return out.view(*shape, self.n)


class W8HeadMethod(G256LinearMethod):
    """The W8 LM head (method.py:65-91): codes uint32 [15520, 128, 4, 16] and
    scales fp16 [248320, 16]; apply runs 64-row slices through head_out."""
    fields = ('head_tilebank_codes', 'head_scales')

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **attrs):
        self.k, self.n = input_size, output_size
        if (input_size_per_partition, input_size, output_size, params_dtype,
                getattr(layer, 'tp_size', 1)) != (2048, 2048, native.HEAD_VOCAB, torch.bfloat16, 1):
            raise ValueError('W8 head requires the full TP1 Ornith vocabulary')
        layer._g256_device = attrs.get('device')
        register_packed(layer, [(self.fields[0], (native.HEAD_VOCAB // 16, 128, 4, 16), torch.uint32),
                                (self.fields[1], (native.HEAD_VOCAB, 16), torch.float16)])

    def apply(self, layer, x, bias=None):
        if self.runtime is None or not layer._g256_ready or bias is not None:
            raise RuntimeError('W8 head requires loaded weights and a bound worker')
        x = x.reshape(-1, self.k).contiguous()
        out = torch.empty((x.shape[0], self.n), dtype=x.dtype, device=x.device)
        for start in range(0, x.shape[0], native.HEAD_ROWS):
            native.head_out(x[start:start + native.HEAD_ROWS], layer.head_tilebank_codes, layer.head_scales,
                            self.runtime.workspace, out[start:start + native.HEAD_ROWS],
                            self.runtime.slots[self.slot], self.runtime.head_geometry)
        return out


class G256MoEMethod:
    """The routed method of one MoE layer (method.py:101-184) on this library.

    `runtime` is an `ornith_b200.runtime.Runtime` (workspace arena, capacity,
    per-layer flag slots) bound with `bind(runtime, slot)`, as the reference's
    worker binds its runtime before the first forward."""

    def __init__(self):
        self.runtime, self.slot = None, None

    def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                       **attrs):
        """Register the N16 banks as the checkpoint stores them (method.py:112-122):
        codes uint32 [256, N/16, K/256, 32, 16], metadata uint32 [256, N/16, K/256, 16]."""
        if (num_experts, hidden_size, intermediate_size_per_partition, params_dtype) != (E, H, I, torch.bfloat16):
            raise ValueError('G256 routed weights require E256/H2048/I512 BF16')
        self.runtime, self.slot = None, None
        layer._ornith_weights_ready = False
        device = attrs.get('device')
        for proj, n, k in PROJECTIONS:
            for suffix, shape in (('codes', (E, n // 16, k // 256, 32, 16)), ('metadata', (E, n // 16, k // 256, 16))):
                layer.register_parameter(f'{proj}_tilebank_{suffix}', torch.nn.Parameter(
                    torch.empty(shape, dtype=torch.uint32, device=device), requires_grad=False))
        install_tilebank_loader(layer)

    def process_weights_after_loading(self, layer):
        require_complete_tilebank_load(layer)
        layer._ornith_weights_ready = True

    def prepare_n32_weights(self, layer, *, replace=False):
        """Reorder the loaded N16 banks once into N32 storage (method.py:124-158):
        codes [E, N/32, K/256, 32, 32] with column c of an N32 tile = 16*half +
        lane of N16 tile 2t+half, metadata [E, N/32, K/256, 32].  replace=True
        swaps each parameter's payload (the checkpoint stays in its load
        format); otherwise the N32 banks are registered as buffers
        `<proj>_n32_<suffix>`.  Returns the bytes of N32 storage."""
        if not layer._ornith_weights_ready or self.runtime is not None:
            raise RuntimeError('N32 shadows require loaded, unbound routed weights')
        if getattr(layer, '_ornith_storage_n32', False):
            raise RuntimeError('N32 expert storage is prepared once')
        total = 0
        with torch.no_grad():
            for proj, n, k in PROJECTIONS:
                if hasattr(layer, f'{proj}_n32_codes') or hasattr(layer, f'{proj}_n32_metadata'):
                    raise RuntimeError('N32 routed shadows are prepared once')
                codes = getattr(layer, f'{proj}_tilebank_codes')
                meta = getattr(layer, f'{proj}_tilebank_metadata')
                for parent in (codes, meta):
                    if (parent.dtype != torch.uint32 or parent.device.type != 'cuda'
                            or not parent.is_contiguous() or parent.shape[1] % 2):
                        raise ValueError('N32 shadows require contiguous GPU U32 N16 banks')
                codes32, meta32 = native.repack_n16_to_n32(codes, meta, n, k)
                for suffix, parent, shadow in (('codes', codes, codes32), ('metadata', meta, meta32)):
                    if replace:
                        parent.data = shadow
                    else:
                        layer.register_buffer(f'{proj}_n32_{suffix}', shadow, persistent=False)
                    total += shadow.numel() * shadow.element_size()
        if replace:
            layer._ornith_storage_n32 = True
        return total

    def bind(self, runtime, slot):
        """Attach the worker's runtime and this layer's flag slot."""
        self.runtime, self.slot = runtime, slot

    def n32_banks(self, layer):
        if getattr(layer, '_ornith_storage_n32', False):
            names = [f'{p}_tilebank_{s}' for p, _, _ in PROJECTIONS for s in ('codes', 'metadata')]
        elif hasattr(layer, 'w13_n32_codes'):
            names = [f'{p}_n32_{s}' for p, _, _ in PROJECTIONS for s in ('codes', 'metadata')]
        else:
            raise RuntimeError('This library computes on N32 storage: call prepare_n32_weights first')
        return [getattr(layer, n) for n in names]

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
        """Routed experts of one layer (method.py:165-183): x bf16 [T, 2048],
        topk_weights fp32 [T, 8], topk_ids int32 [T, 8] (-1 = padding) ->
        a fresh bf16 [T, 2048].  The shared expert is not part of this call
        (its output comes from the shared-expert path, as in the reference)."""
        if self.runtime is None or not layer._ornith_weights_ready:
            raise RuntimeError('G256 routed weights require a bound worker')
        gate, gate_meta, down, down_meta = self.n32_banks(layer)
        out = torch.empty_like(x)
        native.routed_out(x, topk_weights, topk_ids, gate, gate_meta, down, down_meta, self.runtime.workspace, out,
                          self.runtime.slots[self.slot], self.runtime.capacity)
        return out
