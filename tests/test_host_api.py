"""Host contract of dsa_b200.forward on meta tensors (no GPU).

Mirrors the reference's tools/check_host_api.py: the device check is
pointed at "meta" (check_host_api.py:58 does the same for "npu") and the
native launch is replaced by a recording stub (check_host_api.py:23-32);
then the rejection matrix of check_host_api.py:88-129 is replayed. Launch
entries go through the real library's host-side checks
(dsa_check_launch / dsa_default_launch need no GPU).
"""
from dataclasses import replace

import pytest
import torch

import dsa_b200
from dsa_b200 import _native, api, config


def _native_family_union():
    return _native.FAMILY_PAIR_UNION


@pytest.fixture()
def meta_api(monkeypatch):
    events = []
    monkeypatch.setattr(api, "DEVICE_TYPE", "meta")
    monkeypatch.setattr(api, "_default_cache", {})

    def launch(args, stream):
        events.append(("launch", args.batch, args.queries, args.heads, args.length, args.topk,
                       args.launch.family, args.launch.keys_per_tile, args.launch.split,
                       args.workspace_bytes))
        return 2 if args.launch.split > 1 or args.launch.family == _native_family_union() else 1

    monkeypatch.setattr(api, "_launch_native", launch)
    return events


def data_for(shape):
    b, s, h, length, selected = shape
    shapes = [(b, s, h, 512), (b, length, 1, 512), (b, s, h, 64), (b, length, 1, 64), (b, s, 1, selected)]
    return tuple(torch.empty(sh, dtype=torch.int32 if i == 4 else torch.bfloat16, device="meta")
                 for i, sh in enumerate(shapes))


@pytest.mark.parametrize("name", sorted(config.CASE_SHAPES))
def test_allocation_and_launch(meta_api, name):
    shape = config.CASE_SHAPES[name]
    b, s, h, length, k = shape
    (out, mx, sm), kernels = dsa_b200.forward(*data_for(shape), return_kernels=True)
    assert out.shape == (b, s, h, 512) and out.dtype == torch.bfloat16
    assert mx.shape == (b, 1, s, h) and mx.dtype == torch.float32
    assert sm.shape == mx.shape and sm.dtype == torch.float32
    assert len(meta_api) == 1
    split = meta_api[0][8]
    assert len(kernels) == (2 if split > 1 else 1)
    ws = meta_api[0][9]
    if split > 1:
        rows = b * s * split * h
        assert ws >= rows * 514 * 4
    else:
        assert ws == 0


def test_dispatch_is_shape_only(meta_api):
    shape = config.CASE_SHAPES["decode_b8"]
    dsa_b200.forward(*data_for(shape))
    dsa_b200.forward(*data_for(shape))
    assert meta_api[0] == meta_api[1]


def _mutations():
    base_shape = config.CASE_SHAPES["decode_b4_h32"]
    data = data_for(base_shape)
    out = []
    for i, tensor in enumerate(data):
        for sh in (tensor.shape[:-1], tensor.shape[:-1] + (tensor.shape[-1] + 1,), (0,) + tensor.shape[1:]):
            if i == 4 and len(sh) == 4 and sh[-1] == tensor.shape[-1] + 1:
                continue  # a ragged TOPK is a supported shape here (test_ragged_topk_accepted)
            altered = list(data)
            altered[i] = torch.empty(sh, dtype=tensor.dtype, device="meta")
            out.append((f"shape-{i}-{tuple(sh)}", altered, {}, ValueError))
        for kind in ("dtype", "contiguous", "device"):
            altered = list(data)
            if kind == "dtype":
                altered[i] = torch.empty(tensor.shape, dtype=torch.float32, device="meta")
            elif kind == "contiguous":
                altered[i] = torch.empty(tensor.shape[:-1] + (tensor.shape[-1] * 2,),
                                         dtype=tensor.dtype, device="meta")[..., ::2]
            else:
                altered[i] = torch.empty(tensor.shape, dtype=tensor.dtype, device="cpu")
            out.append((f"{kind}-{i}", altered, {}, ValueError))
    for core in (0, -1, True, 1.5, "28"):
        out.append((f"core-{core}", data, {"cores": core}, ValueError))
    base = config.Tuning(16, 32, 4)
    for field, values in {"bm": (0, 8, 64, 16.0), "bn": (0, 127, 128, 256, 32.0),
                          "split": (0, -1, True, 10 ** 6), "pv_cols": (0, 64, 256.0)}.items():
        for value in values:
            out.append((f"tuning-{field}-{value}", data, {"config": replace(base, **{field: value})}, ValueError))
    out.append(("config-type", data, {"config": {}}, TypeError))
    return out


@pytest.mark.parametrize("name,args,kwargs,exc", _mutations(), ids=lambda v: v if isinstance(v, str) else "")
def test_rejections(meta_api, name, args, kwargs, exc):
    with pytest.raises(exc):
        dsa_b200.forward(*args, **kwargs)
    assert meta_api == [], "nothing may launch after a rejected call"


def test_explicit_tuning_accepted(meta_api):
    shape = config.CASE_SHAPES["decode_b4_h32"]
    dsa_b200.forward(*data_for(shape), config=config.Tuning(16, 64, 3))
    assert meta_api[0][7:9] == (64, 3)


def test_unknown_shape_uses_heuristic(meta_api):
    """Deliberate difference from the reference (dsa/api.py:88-92 raises for a
    shape outside its 16-entry table): any shape meeting the input contract
    gets a shape-only launch entry."""
    dsa_b200.forward(*data_for((4, 2, 32, 8192, 2048)))
    assert len(meta_api) == 1


def test_ragged_topk_accepted(meta_api):
    """The reference rejects TOPK=2049 only because that shape is not in its
    table; the kernels here mask the ragged last tile."""
    dsa_b200.forward(*data_for((4, 1, 32, 8192, 2049)))
    assert meta_api[0][5] == 2049


def test_head_count_must_be_multiple_of_16(meta_api):
    with pytest.raises(ValueError):
        dsa_b200.forward(*data_for((1, 1, 24, 1024, 64)))


def test_dsa_package_shim(meta_api):
    """``import dsa; dsa.forward(...)`` works literally, as for the reference
    package (dsa/__init__.py:2-5), and runs this library's forward."""
    import dsa

    assert dsa.forward is dsa_b200.forward
    assert dsa.Tuning is dsa_b200.Tuning
    assert dsa.CASE_SHAPES is dsa_b200.CASE_SHAPES and dsa.SELECTED is dsa_b200.SELECTED
    assert set(dsa.__all__) == {"forward", "Tuning", "CASE_SHAPES", "SELECTED"}
    out, mx, sm = dsa.forward(*data_for((1, 2, 32, 1024, 256)))
    assert out.shape == (1, 2, 32, 512) and mx.shape == (1, 1, 2, 32) and len(meta_api) == 1
