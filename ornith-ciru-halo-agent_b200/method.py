"""Packed-weight methods the reference plugin drives: routed experts, dense
G256 linears and the W8 head, with their strict checkpoint loaders.

The interfaces are the plugin's (plugin-site/ornith_g256/method.py, loader.py),
so that a caller written for it works unchanged; the code is this library's:
  * `G256MoEMethod` (method.py:101-184): create_weights registers the four N16
    tile banks of a routed layer and installs the tile-bank loader,
    process_weights_after_loading seals them, prepare_n32_weights reorders
    them once, on the GPU, into the N32 storage the kernels use, and
    apply(layer, x, topk_weights, topk_ids, shared_experts=None,
    shared_experts_input=None) returns a fresh bf16 output through
    `ornith_b200::routed_out`;
  * the tile-bank loader (loader.py:12-54): `routed_experts.<field>` tensors
    are admitted only for a known field, once, with the registered shape and
    dtype, materialised, and, for metadata, as CPU uint32 fp16 pairs with
    finite values and scales at or above the 2^-14 floor;
  * `register_packed`, `G256LinearMethod`, `W8HeadMethod` (method.py:11-91):
    packed parameters that accept exactly one copy of their shape and dtype
    before sealing; apply through `ornith_b200::dense_out` / `head_out`.
The kernels trust the banks: these admission rules are the only check a
checkpoint gets.  The layer is any torch.nn.Module (vLLM's layers in the
reference); rejected loads raise ValueError, as the plugin's do.
"""
import torch

from . import native

E, H, I = 256, 2048, 512
PREFIX = 'routed_experts.'
# bank name prefix, output columns N, input depth K of the two routed projections
PROJECTIONS = (('w13', 2 * I, H), ('w2', H, I))
FIELDS = tuple(f'{proj}_tilebank_{kind}' for proj, _, _ in PROJECTIONS for kind in ('codes', 'metadata'))
SCALE_FLOOR = 2.0 ** -14


def _metadata_problem(value):
    """Why a metadata tensor cannot be admitted, or None.  Each uint32 word
    holds an fp16 scale (low half) and an fp16 offset (high half)."""
    if value.device.type != 'cpu' or value.dtype != torch.uint32:
        return 'metadata must arrive as CPU uint32 words'
    halves = value.contiguous().view(torch.float16).view(*value.shape, 2)
    if not bool(torch.isfinite(halves).all()):
        return 'metadata holds a non-finite scale or offset'
    if not bool((halves[..., 0] >= SCALE_FLOOR).all()):
        return 'metadata holds a scale below 2^-14'
    return None


class _TilebankLoader:
    """layer.load_weights for the routed banks: a generator over (name,
    tensor) pairs that yields each admitted name after copying it."""

    def __init__(self, layer):
        self.layer = layer
        self.loaded = set()

    def __call__(self, weights):
        layer = self.layer
        if getattr(layer, '_ornith_weights_ready', False):
            raise ValueError('tile banks are sealed; no further loads')
        for key, value in weights:
            field = key[len(PREFIX):] if key.startswith(PREFIX) else None
            if field not in FIELDS:
                raise ValueError(f'not a routed tile-bank field: {key}')
            if field in self.loaded:
                raise ValueError(f'{field} loaded twice')
            target = layer._parameters.get(field)
            if target is None:
                raise ValueError(f'no registered parameter for {field}')
            if (value.shape, value.dtype) != (target.shape, target.dtype):
                raise ValueError(f'{field}: expected {tuple(target.shape)} {target.dtype}, '
                                 f'got {tuple(value.shape)} {value.dtype}')
            if 'meta' in (value.device.type, target.device.type):
                raise ValueError(f'{field}: meta tensors cannot be loaded')
            if field.endswith('_metadata'):
                problem = _metadata_problem(value)
                if problem:
                    raise ValueError(f'{field}: {problem}')
            with torch.no_grad():
                target.copy_(value)
            self.loaded.add(field)
            yield key


def install_tilebank_loader(layer):
    """Attach the tile-bank loader; once, after the four banks are registered."""
    if isinstance(getattr(layer, 'load_weights', None), _TilebankLoader):
        raise ValueError('tile-bank loader installed twice')
    missing = [f for f in FIELDS if f not in layer._parameters]
    if missing:
        raise ValueError(f'register the tile-bank parameters before the loader (missing {missing})')
    layer.load_weights = _TilebankLoader(layer)


def require_complete_tilebank_load(layer):
    """Raise unless all four routed banks were loaded."""
    loader = getattr(layer, 'load_weights', None)
    loaded = loader.loaded if isinstance(loader, _TilebankLoader) else set()
    missing = sorted(set(FIELDS) - loaded)
    if missing:
        raise ValueError(f'tile-bank checkpoint incomplete: missing {missing}')


class _PackedLoad:
    """weight_loader of one packed parameter: exactly one copy of its shape
    and dtype, into that parameter, before the layer is sealed."""

    def __init__(self, layer, name, param):
        self.layer, self.name, self.param = layer, name, param

    def __call__(self, destination, value, *shard_args):
        layer, name, param = self.layer, self.name, self.param
        if destination is not param:
            raise ValueError(f'packed field {name}: the loader was given another parameter')
        if layer._g256_ready or name in layer._g256_loaded:
            raise ValueError(f'packed field {name}: second load or load after sealing')
        if (value.shape, value.dtype) != (param.shape, param.dtype):
            raise ValueError(f'packed field {name}: expected {tuple(param.shape)} {param.dtype}, '
                             f'got {tuple(value.shape)} {value.dtype}')
        with torch.no_grad():
            param.copy_(value)
        layer._g256_loaded.add(name)


def register_packed(layer, specs, device=None):
    """Register packed parameters, (name, shape, dtype) each, with their loaders."""
    layer._g256_loaded = set()
    layer._g256_ready = False
    for name, shape, dtype in specs:
        param = torch.nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)
        layer.register_parameter(name, param)
        param.weight_loader = _PackedLoad(layer, name, param)


class G256LinearMethod:
    """A dense G256 linear: codes uint32 [N/16, K/256, 32, 16] and metadata
    uint32 [N/16, K/256, 16]; apply(x [..., K]) -> bf16 [..., N]."""
    fields = ('g256_codes', 'g256_metadata')

    def __init__(self, prefix=''):
        self.prefix, self.runtime, self.slot = prefix, None, None

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **attrs):
        self.k, self.n = input_size, output_size
        problems = [why for bad, why in (
            (input_size_per_partition != input_size, 'a split input'),
            (sum(output_partition_sizes) != output_size, 'output partitions that do not sum to the output'),
            (getattr(layer, 'tp_size', 1) != 1, 'tensor parallelism'),
            (params_dtype != torch.bfloat16, f'dtype {params_dtype}'),
            (getattr(layer, 'has_bias', False), 'a bias'),
            (not 0 < output_size <= 12288 or output_size % 16, f'N = {output_size} (1..12288, a multiple of 16)'),
            (not 0 < input_size <= 8192 or input_size % 256, f'K = {input_size} (1..8192, a multiple of 256)'),
        ) if bad]
        if problems:
            raise ValueError(f'G256 linear {self.prefix}: unsupported geometry: {"; ".join(problems)}')
        register_packed(layer, [(self.fields[0], (self.n // 16, self.k // 256, 32, 16), torch.uint32),
                                (self.fields[1], (self.n // 16, self.k // 256, 16), torch.uint32)],
                        attrs.get('device'))

    def process_weights_after_loading(self, layer):
        missing = sorted(set(self.fields) - layer._g256_loaded)
        if missing:
            raise ValueError(f'{self.prefix}: packed weights not loaded: {missing}')
        layer._g256_ready = True

    def bind(self, runtime, slot):
        """Attach the worker's runtime and this layer's flag slot."""
        self.runtime, self.slot = runtime, slot

    def _check_ready(self, layer, bias):
        if self.runtime is None or not layer._g256_ready or bias is not None:
            raise RuntimeError(f'{self.prefix}: apply needs sealed weights and a bound runtime, and takes no bias')

    def apply(self, layer, x, bias=None):
        self._check_ready(layer, bias)
        lead = x.shape[:-1]
        rows = x.reshape(-1, self.k).contiguous()
        out = torch.empty((rows.shape[0], self.n), dtype=rows.dtype, device=rows.device)
        rt = self.runtime
        native.dense_out(rows, layer.g256_codes, layer.g256_metadata, rt.workspace, out, rt.slots[self.slot],
                         rt.capacity, self.n, self.k, rt.dense_geometry, rt.dense_a8_max_rows)
        return out.view(*lead, self.n)


class W8HeadMethod(G256LinearMethod):
    """The W8 LM head: codes uint32 [15520, 128, 4, 16] and scales fp16
    [248320, 16]; apply runs the rows through head_out 64 at a time."""
    fields = ('head_tilebank_codes', 'head_scales')

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **attrs):
        self.k, self.n = input_size, output_size
        want = (2048, 2048, native.HEAD_VOCAB, torch.bfloat16, 1)
        got = (input_size_per_partition, input_size, output_size, params_dtype, getattr(layer, 'tp_size', 1))
        if got != want:
            raise ValueError(f'W8 head needs K 2048 and the full TP1 Ornith vocabulary of {native.HEAD_VOCAB} '
                             f'in bf16, got {got}')
        register_packed(layer, [(self.fields[0], (native.HEAD_VOCAB // 16, 128, 4, 16), torch.uint32),
                                (self.fields[1], (native.HEAD_VOCAB, 16), torch.float16)], attrs.get('device'))

    def apply(self, layer, x, bias=None):
        self._check_ready(layer, bias)
        rows = x.reshape(-1, self.k).contiguous()
        out = torch.empty((rows.shape[0], self.n), dtype=rows.dtype, device=rows.device)
        rt, step = self.runtime, native.HEAD_ROWS
        for first in range(0, rows.shape[0], step):
            native.head_out(rows[first:first + step], layer.head_tilebank_codes, layer.head_scales, rt.workspace,
                            out[first:first + step], rt.slots[self.slot], rt.head_geometry)
        return out.view(*x.shape[:-1], self.n)


class G256MoEMethod:
    """The routed method of one MoE layer on this library.  `runtime` is an
    ornith_b200 Runtime (workspace arena, capacity, per-layer flag slots)
    attached with bind(runtime, slot) before the first apply."""

    def __init__(self):
        self.runtime, self.slot = None, None

    def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                       **attrs):
        """Register the N16 banks in the checkpoint's layout: codes uint32
        [256, N/16, K/256, 32, 16] and metadata uint32 [256, N/16, K/256, 16]."""
        if (num_experts, hidden_size, intermediate_size_per_partition, params_dtype) != (E, H, I, torch.bfloat16):
            raise ValueError(f'routed G256 banks are fixed at {E} experts, hidden {H}, intermediate {I}, bf16; '
                             f'got {(num_experts, hidden_size, intermediate_size_per_partition, params_dtype)}')
        self.runtime, self.slot = None, None
        layer._ornith_weights_ready = False
        device = attrs.get('device')
        for proj, n, k in PROJECTIONS:
            shapes = {'codes': (E, n // 16, k // 256, 32, 16), 'metadata': (E, n // 16, k // 256, 16)}
            for kind, shape in shapes.items():
                bank = torch.empty(shape, dtype=torch.uint32, device=device)
                layer.register_parameter(f'{proj}_tilebank_{kind}', torch.nn.Parameter(bank, requires_grad=False))
        install_tilebank_loader(layer)

    def process_weights_after_loading(self, layer):
        require_complete_tilebank_load(layer)
        layer._ornith_weights_ready = True

    def prepare_n32_weights(self, layer, *, replace=False):
        """Reorder the loaded N16 banks once into N32 storage on the GPU
        (column 16h + l of N32 tile t is column l of N16 tile 2t + h; the
        reference does it with a torch permute, method.py:124-158).
        replace=True swaps each parameter's payload in place; otherwise the N32
        banks become buffers `<proj>_n32_<kind>`.  Returns the N32 bytes."""
        if not layer._ornith_weights_ready or self.runtime is not None:
            raise RuntimeError('reorder to N32 storage after loading and before binding')
        if getattr(layer, '_ornith_storage_n32', False) or hasattr(layer, 'w13_n32_codes'):
            raise RuntimeError('N32 storage was already prepared for this layer')
        reordered = []
        for proj, n, k in PROJECTIONS:
            codes = getattr(layer, f'{proj}_tilebank_codes')
            meta = getattr(layer, f'{proj}_tilebank_metadata')
            if any(b.dtype != torch.uint32 or b.device.type != 'cuda' or not b.is_contiguous() or b.shape[1] % 2
                   for b in (codes, meta)):
                raise ValueError('the N32 reorder needs contiguous CUDA uint32 N16 banks')
            with torch.no_grad():
                codes32, meta32 = native.repack_n16_to_n32(codes, meta, n, k)
            reordered += [(proj, 'codes', codes, codes32), (proj, 'metadata', meta, meta32)]
        for proj, kind, bank, n32 in reordered:
            if replace:
                bank.data = n32
            else:
                layer.register_buffer(f'{proj}_n32_{kind}', n32, persistent=False)
        if replace:
            layer._ornith_storage_n32 = True
        return sum(n32.numel() * n32.element_size() for *_, n32 in reordered)

    def bind(self, runtime, slot):
        """Attach the worker's runtime and this layer's flag slot."""
        self.runtime, self.slot = runtime, slot

    def n32_banks(self, layer):
        """(gate codes, gate metadata, down codes, down metadata) in N32 storage."""
        if getattr(layer, '_ornith_storage_n32', False):
            names = FIELDS
        elif hasattr(layer, 'w13_n32_codes'):
            names = tuple(f'{proj}_n32_{kind}' for proj, _, _ in PROJECTIONS for kind in ('codes', 'metadata'))
        else:
            raise RuntimeError('N32 storage missing: call prepare_n32_weights first')
        return [getattr(layer, name) for name in names]

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
        """x bf16 [T, 2048], topk_weights fp32 [T, 8], topk_ids int32 [T, 8]
        (-1 = padding) -> a fresh bf16 [T, 2048].  The shared expert is not
        part of this call: its output comes from the shared-expert path."""
        if self.runtime is None or not layer._ornith_weights_ready:
            raise RuntimeError('apply needs loaded routed weights and a bound runtime')
        out = torch.empty_like(x)
        rt = self.runtime
        native.routed_out(x, topk_weights, topk_ids, *self.n32_banks(layer), rt.workspace, out, rt.slots[self.slot],
                          rt.capacity)
        return out
