"""Host side of the widened boundary (no GPU): scale validation and its path
to the C ABI, the vendor-operator shaped wrapper's argument rules, and the
oracle's scale / no-valid-index semantics."""
import math

import pytest
import torch

import dsa_b200
from dsa_b200 import api
from oracle import sparse_mla as oracle


@pytest.fixture()
def recorded(monkeypatch):
    calls = []
    monkeypatch.setattr(api, "DEVICE_TYPE", "meta")
    monkeypatch.setattr(api, "_default_cache", {})

    def launch(args, stream):
        calls.append(args.scale)
        return 1

    monkeypatch.setattr(api, "_launch_native", launch)
    return calls


def meta_data(b=1, s=2, h=16, length=256, k=64):
    shapes = [(b, s, h, 512), (b, length, 1, 512), (b, s, h, 64), (b, length, 1, 64), (b, s, 1, k)]
    return tuple(torch.empty(sh, dtype=torch.int32 if i == 4 else torch.bfloat16, device="meta")
                 for i, sh in enumerate(shapes))


def test_scale_values(recorded):
    data = meta_data()
    dsa_b200.forward(*data)
    dsa_b200.forward(*data, scale=0.125)
    dsa_b200.forward(*data, scale=0.5)
    assert recorded == [0.0, 0.125, 0.5]


@pytest.mark.parametrize("bad", [0, 0.0, -0.1, 0.51, 1, float("nan"), float("inf"), True, "0.1", [0.1]])
def test_scale_rejected(recorded, bad):
    with pytest.raises(ValueError):
        dsa_b200.forward(*meta_data(), scale=bad)
    assert recorded == []


def test_plan_scale_rejected(recorded):
    with pytest.raises(ValueError):
        dsa_b200.ForwardPlan(*meta_data(), scale=2.0)


@pytest.mark.parametrize("kwargs,message", [
    ({"attention_mode": 0}, "attention_mode"),
    ({"sparse_mode": 3}, "sparse_mode"),
    ({"layout_query": "TND"}, "layout"),
    ({"layout_kv": "PA_BSND"}, "layout"),
    ({"sparse_block_size": 4}, "sparse_block_size"),
    ({"block_table": torch.zeros(1)}, "block_table"),
    ({"actual_seq_lengths_kv": [256]}, "ragged"),
    ({"actual_seq_lengths_query": [2]}, "ragged"),
    ({"query_rope": None}, "rope"),
])
def test_vendor_wrapper_rejects_unsupported(recorded, kwargs, message):
    q, kv, qr, kr, ids = meta_data()
    call = dict(query_rope=qr, key_rope=kr)
    call.update(kwargs)
    with pytest.raises(ValueError, match=message):
        dsa_b200.sparse_flash_attention(q, kv, kv, ids, 0.1, **call)
    assert recorded == []


def test_vendor_wrapper_value_must_be_key(recorded):
    q, kv, qr, kr, ids = meta_data()
    other = torch.empty_like(kv)
    with pytest.raises(ValueError, match="same tensor"):
        dsa_b200.sparse_flash_attention(q, kv, other, ids, 0.1, query_rope=qr, key_rope=kr)
    with pytest.raises(ValueError, match="scale_value"):
        dsa_b200.sparse_flash_attention(q, kv, kv, ids, None, query_rope=qr, key_rope=kr)


def test_vendor_wrapper_forwards_scale_and_outputs(recorded):
    q, kv, qr, kr, ids = meta_data()
    out, mx, sm = dsa_b200.npu_sparse_flash_attention(q, kv, kv, ids, 576 ** -0.5, query_rope=qr, key_rope=kr,
                                                      attention_mode=2, sparse_mode=0,
                                                      return_softmax_lse=True)
    assert recorded == [pytest.approx(1 / 24)]
    assert out.shape == q.shape and mx.shape == (1, 1, 2, 16) and sm.shape == mx.shape
    out, mx, sm = dsa_b200.sparse_flash_attention(q, kv, kv, ids, 0.25, query_rope=qr, key_rope=kr)
    assert mx.numel() == 0 and sm.numel() == 0 and recorded[-1] == 0.25


def test_oracle_scale_matches_default_at_one_24th():
    data = oracle.make_inputs((1, 2, 4, 128, 16), 1, "normal")
    a = oracle.reference_forward(*data)
    b = oracle.reference_forward(*data, scale=1 / 24)
    m = oracle.accuracy(b, a)
    assert m["output"]["max_normalized"] < 1e-6 and m["maximum"]["max_normalized"] < 1e-6


def test_oracle_scale_is_applied():
    q, kv, qr, kr, ids = oracle.make_inputs((1, 1, 2, 64, 8), 2, "normal")
    _, mx, sm = oracle.reference_forward(q, kv, qr, kr, ids, scale=0.3)
    idx = ids[0, 0, 0].long()
    s = (q[0, 0].float() @ kv[0, idx, 0].float().T + qr[0, 0].float() @ kr[0, idx, 0].float().T) * 0.3
    torch.testing.assert_close(mx[0, 0, 0], s.amax(-1), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(sm[0, 0, 0], (s - s.amax(-1, keepdim=True)).exp().sum(-1), rtol=1e-6, atol=1e-6)


def test_oracle_defined_invalid_rows():
    q, kv, qr, kr, ids = oracle.make_inputs((1, 3, 2, 64, 8), 4, "normal")
    ids[0, 1] = -1
    out, mx, sm = oracle.reference_forward(q, kv, qr, kr, ids, defined_invalid=True)
    assert torch.equal(out[0, 1], torch.zeros_like(out[0, 1]))
    assert bool(torch.isneginf(mx[0, 0, 1]).all()) and torch.equal(sm[0, 0, 1], torch.zeros(2))
    ref = oracle.reference_forward(q, kv, qr, kr, ids)
    assert bool(torch.isnan(ref[0][0, 1]).all())  # the reference's own math leaves it undefined
    for t, r in zip((out, mx, sm), ref):
        keep = [0, 2]
        if t.dim() == 4 and t.shape[1] == 1:
            assert torch.equal(t[:, :, keep], r[:, :, keep])
        else:
            assert torch.equal(t[:, keep], r[:, keep])
    assert math.isinf(float(mx[0, 0, 1, 0]))
