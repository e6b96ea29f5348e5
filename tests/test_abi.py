"""libvqmoe.so loads, exports every symbol include/vqmoe.h declares, and its
host-only entry points answer without a GPU (CPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from knurlogic_b200 import _lib, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "vqmoe.h"


@pytest.fixture(scope="module")
def so():
    build.build()
    return _lib.lib()


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"VQMOE_API\s+[\w\s\*]+?\b(vqmoe_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported(so):
    names = declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(so, n), n
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(names) == bound, set(names) ^ bound


def test_abi_version_and_struct_layout(so):
    assert so.vqmoe_abi_version() == 4
    # vqmoe_linear: 4 int32, 4 pointers, 4 int32 (the last: the activation),
    # the affine biases pointer, bits, a reserved word
    assert ctypes.sizeof(_lib.Linear) == 16 + 4 * 8 + 16 + 8 + 8
    # vqmoe_block: ..., 4 shared pointers, router_mode, wait_polls
    assert ctypes.sizeof(_lib.Block) == 16 + 8 + 3 * ctypes.sizeof(_lib.Linear) + 4 * 8 + 8


def _block(H=2048, E=128, k=8, I=768, Is=768):
    b = _lib.Block(hidden=H, num_experts=E, top_k=k, shared_inter=Is)
    for name, out, inp in (("gate", I, H), ("up", I, H), ("down", H, I)):
        setattr(b, name, _lib.Linear(format=_lib.FMT_VQ_U8, num_experts=E,
                                     out_features=out, in_features=inp,
                                     codebook_size=256, dim=4, group_size=64))
    return b


def test_workspace_queries_are_host_only(so):
    b = _block()
    n64 = so.vqmoe_block_workspace_size(ctypes.byref(b), 64)
    n128 = so.vqmoe_block_workspace_size(ctypes.byref(b), 128)
    assert 0 < n64 < n128 and n64 % 256 == 0
    # act [T*k, I] + ybuf [T*k, H] dominate
    assert n64 >= 64 * 8 * (768 + 2048) * 2
    g, d = b.gate, b.down
    nglu = so.vqmoe_switch_glu_workspace_size(ctypes.byref(g), ctypes.byref(d), 64, 8)
    assert nglu >= 64 * 8 * 768 * 2 + 64 * 2048 * 2       # act + fp16 copy of x
    nlin = so.vqmoe_switch_linear_workspace_size(ctypes.byref(g), 64, 8, 0)
    assert 0 < nlin < nglu
    assert so.vqmoe_router_workspace_size(64, 128) >= 64 * 129 * 4


def test_bad_arguments_return_a_status_not_a_crash(so):
    b = _block()
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), None, 64, None, 0, None, 0, None)
    assert st != 0
    assert so.vqmoe_last_error()
    b.gate.group_size = 32
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), None, 64, None, 0, None, 0, None)
    assert _lib.STATUS[st] == "BAD_FORMAT"
    assert b"group_size" in so.vqmoe_last_error()
    st = so.vqmoe_prepare_vq(None, None, 2, 32, 100, None, None, None)
    assert _lib.STATUS[st] == "BAD_SHAPE"          # IN not a multiple of 64
    assert _lib.vq_layout_bytes(2, 48, 320) == (2 * 2 * 2 * 2048, 2 * 2 * 2 * 128 * 2)
    b = _block()
    b.wait_polls = -1
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), None, 64, None, 0, None, 0, None)
    assert _lib.STATUS[st] == "BAD_SHAPE" and b"wait_polls" in so.vqmoe_last_error()
    assert _lib.STATUS[so.vqmoe_workspace_status(None, None)] == "BAD_POINTER"
