"""CPU: the routed method's weight registration and the strict tile-bank
loader (plugin-site/ornith_g256/method.py:101-158, loader.py:12-54)."""
import importlib

import pytest
import torch

PREFIX = 'routed_experts.'


@pytest.fixture(scope='module')
def M():
    return importlib.import_module('ornith_b200.method')


def _valid(shape_meta):
    """uint32 metadata words with scale 1.0 (0x3C00) and offset -8.0 (0xC800)."""
    return torch.full(shape_meta, 0x3C00 | (0xC800 << 16), dtype=torch.int64).to(torch.uint32)


def _s32(word):
    """A uint32 bit pattern as the int32 with the same bits."""
    return word - (1 << 32) if word >= 1 << 31 else word


def _layer(M):
    layer = torch.nn.Module()
    method = M.G256MoEMethod()
    method.create_weights(layer, 256, 2048, 512, torch.bfloat16)
    return layer, method


def _checkpoint(layer):
    state = []
    for name in ('w13_tilebank_codes', 'w13_tilebank_metadata', 'w2_tilebank_codes', 'w2_tilebank_metadata'):
        p = getattr(layer, name)
        value = _valid(p.shape) if name.endswith('metadata') else torch.zeros(p.shape, dtype=torch.uint32)
        state.append((PREFIX + name, value))
    return state


def test_create_weights_registers_n16_banks(M):
    layer, _ = _layer(M)
    assert layer.w13_tilebank_codes.shape == (256, 64, 8, 32, 16)
    assert layer.w13_tilebank_metadata.shape == (256, 64, 8, 16)
    assert layer.w2_tilebank_codes.shape == (256, 128, 2, 32, 16)
    assert layer.w2_tilebank_metadata.shape == (256, 128, 2, 16)
    assert all(getattr(layer, n).dtype == torch.uint32 and not getattr(layer, n).requires_grad for n in M.FIELDS)
    with pytest.raises(ValueError, match='fixed at 256 experts'):
        M.G256MoEMethod().create_weights(torch.nn.Module(), 128, 2048, 512, torch.bfloat16)
    with pytest.raises(ValueError, match='installed twice'):
        M.install_tilebank_loader(layer)
    with pytest.raises(ValueError, match='register the tile-bank parameters'):
        M.install_tilebank_loader(torch.nn.Module())


def test_complete_load_seals_the_layer(M):
    layer, method = _layer(M)
    ckpt = _checkpoint(layer)
    names = list(layer.load_weights(iter(ckpt)))
    assert names == [k for k, _ in ckpt]
    assert torch.equal(layer.w2_tilebank_metadata, ckpt[3][1])
    method.process_weights_after_loading(layer)
    assert layer._ornith_weights_ready
    with pytest.raises(ValueError, match='sealed'):
        list(layer.load_weights(iter(ckpt[:1])))


def test_incomplete_load_is_rejected(M):
    layer, method = _layer(M)
    list(layer.load_weights(iter(_checkpoint(layer)[:3])))
    with pytest.raises(ValueError, match='incomplete'):
        method.process_weights_after_loading(layer)


@pytest.mark.parametrize('case', ['unknown', 'prefix', 'duplicate', 'shape', 'dtype', 'meta_device',
                                  'nonfinite_offset', 'nan_scale', 'scale_floor'])
def test_loader_rejects_malformed_checkpoints(M, case):
    layer, _ = _layer(M)
    ckpt = _checkpoint(layer)
    meta = ckpt[1][1].clone()
    if case == 'unknown':
        ckpt.append((PREFIX + 'w13_tilebank_scales', meta))
    elif case == 'prefix':
        ckpt[0] = ('experts.w13_tilebank_codes', ckpt[0][1])
    elif case == 'duplicate':
        ckpt.append(ckpt[0])
    elif case == 'shape':
        ckpt[2] = (ckpt[2][0], ckpt[2][1][:255])
    elif case == 'dtype':
        ckpt[0] = (ckpt[0][0], ckpt[0][1].view(torch.int32))
    elif case == 'meta_device':
        ckpt[1] = (ckpt[1][0], torch.empty(meta.shape, dtype=torch.uint32, device='meta'))
    else:
        words = meta.view(torch.int32)
        if case == 'nonfinite_offset':
            words[3, 1, 2, 5] = _s32(0x3C00 | (0x7C00 << 16))          # offset +inf
        elif case == 'nan_scale':
            words[0, 0, 0, 0] = _s32(0x7E00 | (0xC800 << 16))          # scale NaN
        else:
            words[255, 63, 7, 15] = _s32(0x0200 | (0xC800 << 16))      # subnormal scale < 2^-14
        ckpt[1] = (ckpt[1][0], meta)
    with pytest.raises(ValueError):
        list(layer.load_weights(iter(ckpt)))


def test_method_needs_binding_and_gpu_banks(M):
    layer, method = _layer(M)
    list(layer.load_weights(iter(_checkpoint(layer))))
    method.process_weights_after_loading(layer)
    x = torch.zeros((1, 2048), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match='bound runtime'):
        method.apply(layer, x, torch.zeros((1, 8)), torch.zeros((1, 8), dtype=torch.int32))
    with pytest.raises(ValueError, match='CUDA uint32 N16'):
        method.prepare_n32_weights(layer)
    unloaded, m2 = _layer(M)
    with pytest.raises(AttributeError):
        m2.prepare_n32_weights(torch.nn.Module())
    with pytest.raises(RuntimeError, match='after loading and before binding'):
        m2.prepare_n32_weights(unloaded)


def test_dense_linear_registration_and_loader(M):
    layer = torch.nn.Module()
    method = M.G256LinearMethod('model.layers.0.linear_attn.in_proj_qkvz')
    method.create_weights(layer, 2048, [12288], 2048, 12288, torch.bfloat16)
    assert layer.g256_codes.shape == (768, 8, 32, 16) and layer.g256_metadata.shape == (768, 8, 16)
    for bad in [dict(input_size_per_partition=1024), dict(output_size=12304), dict(input_size=2100),
                dict(params_dtype=torch.float16)]:
        args = dict(input_size_per_partition=2048, output_partition_sizes=[12288], input_size=2048,
                    output_size=12288, params_dtype=torch.bfloat16)
        args.update(bad)
        if 'input_size' in bad:
            args['input_size_per_partition'] = bad['input_size']
        if 'output_size' in bad:
            args['output_partition_sizes'] = [bad['output_size']]
        with pytest.raises(ValueError, match='unsupported geometry'):
            M.G256LinearMethod('x').create_weights(torch.nn.Module(), **args)
    codes = torch.zeros(layer.g256_codes.shape, dtype=torch.uint32)
    with pytest.raises(ValueError, match='expected'):
        layer.g256_codes.weight_loader(layer.g256_codes, codes[:1])
    with pytest.raises(ValueError, match='another parameter'):
        layer.g256_codes.weight_loader(layer.g256_metadata, codes)       # wrong destination
    layer.g256_codes.weight_loader(layer.g256_codes, codes)
    with pytest.raises(ValueError, match='second load'):
        layer.g256_codes.weight_loader(layer.g256_codes, codes)
    with pytest.raises(ValueError, match='not loaded'):
        method.process_weights_after_loading(layer)
    layer.g256_metadata.weight_loader(layer.g256_metadata, _valid(layer.g256_metadata.shape))
    method.process_weights_after_loading(layer)
    with pytest.raises(ValueError, match='after sealing'):
        layer.g256_metadata.weight_loader(layer.g256_metadata, _valid(layer.g256_metadata.shape))
    with pytest.raises(RuntimeError, match='bound runtime'):
        method.apply(layer, torch.zeros((1, 2048), dtype=torch.bfloat16))


def test_w8_head_registration(M):
    layer = torch.nn.Module()
    M.W8HeadMethod('lm_head').create_weights(layer, 2048, [248320], 2048, 248320, torch.bfloat16, device='meta')
    assert layer.head_tilebank_codes.shape == (15520, 128, 4, 16) and layer.head_tilebank_codes.dtype == torch.uint32
    assert layer.head_scales.shape == (248320, 16) and layer.head_scales.dtype == torch.float16
    with pytest.raises(ValueError, match='full TP1 Ornith vocabulary'):
        M.W8HeadMethod('lm_head').create_weights(torch.nn.Module(), 2048, [151936], 2048, 151936, torch.bfloat16)


def test_runtime_settings_are_checked():
    R = importlib.import_module('ornith_b200.runtime')
    with pytest.raises(ValueError, match='32 or 64'):
        R.Runtime(['a'], 8, 'cpu', {'dense_a8_max_rows': 16})
    with pytest.raises(ValueError, match='geometry'):
        R.Runtime(['a'], 8, 'cpu', {'head_geometry': 3})
    rt = R.Runtime(['a', 'b'], 8, 'cpu', dense_shapes=[(12288, 2048), (2048, 4096)])
    native = importlib.import_module('ornith_b200.native')
    assert rt.workspace.numel() >= native.dense_workspace_bytes(8, [(12288, 2048), (2048, 4096)])
    assert rt.dense_geometry == 2 and rt.dense_a8_max_rows == 32 and len(rt.slots) == 2
