"""Host-side checks of Engine that need no GPU: the K/V cache validation the batched calls run for
every request, and its memo of caches that passed before (an Engine shell on the CPU; no library
call is made)."""

import pytest
import torch

from fast_dllm_relax_b200.config import TINY
from fast_dllm_relax_b200.engine import Engine


def _shell() -> Engine:
    eng = Engine.__new__(Engine)
    eng.cfg, eng.dtype, eng.device, eng._h, eng._cache_ok = TINY, torch.float32, torch.device("cpu"), None, {}
    return eng


def test_cache_validation_is_remembered_by_identity():
    eng = _shell()
    k, v = eng.new_cache(64)
    assert eng._cache(k, v) == 64
    assert id(k) in eng._cache_ok
    assert eng._cache(k, v) == 64  # the memo answers
    k2, v2 = eng.new_cache(96)
    assert eng._cache(k2, v2) == 96


def test_remembered_cache_is_checked_again_after_a_change():
    eng = _shell()
    k, v = eng.new_cache(64)
    eng._cache(k, v)
    shape = list(k.shape)
    shape[2] = 96
    k.resize_(shape)  # same object, new capacity: the memo must not answer with the old one
    with pytest.raises(ValueError, match="differ in shape"):
        eng._cache(k, v)
    v.resize_(shape)
    assert eng._cache(k, v) == 96
    bad = torch.empty(shape, dtype=torch.float64)
    with pytest.raises(ValueError, match="model dtype"):
        eng._cache(k, bad)  # a remembered k with another v is checked in full


def test_cache_validation_rejects_bad_layouts():
    eng = _shell()
    c = TINY
    with pytest.raises(ValueError, match="KV cache must be"):
        eng._cache(torch.empty(c.num_hidden_layers, 64, c.num_key_value_heads, c.head_dim),
                   torch.empty(c.num_hidden_layers, 64, c.num_key_value_heads, c.head_dim))
    k, v = eng.new_cache(64)
    with pytest.raises(ValueError, match="contiguous"):
        eng._cache(k.transpose(3, 4).contiguous().transpose(3, 4), v)


def test_confidence_static_rejects_outputs_it_cannot_write():
    """The allocation-free confidence writes ids / maxp through raw device pointers, so host
    tensors, tensors on another device, strided views and wrong dtypes are refused before any
    library call (the shell's device is cuda:0; nothing is launched)."""
    eng = _shell()
    eng.device, eng.dtype = torch.device("cuda", 0), torch.bfloat16
    h = torch.empty((4, TINY.hidden_size), dtype=torch.bfloat16)
    ids, maxp = torch.empty(4, dtype=torch.int32), torch.empty(4, dtype=torch.float32)
    with pytest.raises(ValueError, match="ids must be a contiguous torch.int32 tensor on cuda:0"):
        eng.confidence_static(h, ids, maxp)  # host ids
    meta_ids = torch.empty(4, dtype=torch.int32, device="meta")
    with pytest.raises(ValueError, match="ids must be"):
        eng.confidence_static(h, meta_ids, maxp)  # another device
    eng.device = torch.device("cpu")  # a shell whose device the CPU tensors match: layout checks
    eng.dtype = torch.bfloat16
    with pytest.raises(ValueError, match="ids must be"):
        eng.confidence_static(h, torch.empty(8, dtype=torch.int32)[::2], maxp)  # strided view
    with pytest.raises(ValueError, match="maxp must be"):
        eng.confidence_static(h, ids, torch.empty(4, dtype=torch.float64))  # wrong dtype
    with pytest.raises(ValueError, match="at least rows elements"):
        eng.confidence_static(h, ids[:2], maxp)  # too short
