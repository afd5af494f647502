"""The C-ABI library loads, exports every function include/prism_b200.h declares,
and rejects bad arguments before touching the GPU (no CUDA device needed)."""
import ctypes
import re
from pathlib import Path

import pytest

import prism_test_b200 as pb
from prism_test_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "prism_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"PRISM_API\s+[\w\s\*]+?\b(prism_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    from prism_test_b200 import build
    build.build()
    return _lib.load()


def test_header_declares_expected_functions():
    names = declared_functions()
    assert set(names) == set(_lib.SIGNATURES), names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_abi_version(lib):
    assert lib.prism_abi_version() == 1


def test_workspace_size(lib):
    # status block (256 B) + fp32 scores (rows padded to 4 floats, block to 256 B)
    # + per-row u64 candidate buffers (min(n, 16384) entries)
    assert lib.prism_einsum_topk_workspace_size(1, 32, 1, 131072, 4096, 0) == 256 + 32 * 131072 * 4 + 32 * 16384 * 8
    assert lib.prism_einsum_topk_workspace_size(1, 4, 2, 5, 3, 0) == 256 + 256 + 8 * 5 * 8
    assert lib.prism_topk_merge_workspace_size(6, 1536) == 6 * 1536 * 8
    assert lib.prism_einsum_topk_workspace_size(0, 4, 2, 5, 3, 0) == 0
    assert lib.prism_einsum_topk_workspace_size(1, 4, 2, 5, 3, 7) == 0


def _call(lib, **over):
    args = dict(q=16, k=16, inv=None, dtype=0, B=1, Hq=4, Hkv=2, Sq=1, Sk=256, D=128,
                qs=(512, 128, 128, 1), ks=(65536, 32768, 128, 1), pos=0, causal=-1,
                topk=8, mode=0, base=0, oi=16, os=None, ws=256, wsb=1 << 20, stream=None)
    args.update(over)
    return lib.prism_einsum_topk(
        args["q"], args["k"], args["inv"], args["dtype"], args["B"], args["Hq"], args["Hkv"],
        args["Sq"], args["Sk"], args["D"], _lib.i64_array(args["qs"]), _lib.i64_array(args["ks"]),
        args["pos"], args["causal"], args["topk"], args["mode"], args["base"], args["oi"], args["os"],
        args["ws"], args["wsb"], args["stream"])


@pytest.mark.parametrize("over,code", [
    (dict(q=None), _lib.PRISM_E_INVALID),
    (dict(dtype=5), _lib.PRISM_E_INVALID),
    (dict(Hq=6, Hkv=4), _lib.PRISM_E_INVALID),
    (dict(D=64, qs=(256, 64, 64, 1), ks=(32768, 16384, 64, 1)), _lib.PRISM_E_UNSUPPORTED),
    (dict(ks=(65536, 32768, 256, 1)), _lib.PRISM_E_INVALID),       # rows not contiguous
    (dict(qs=(512, 128, 128, 2)), _lib.PRISM_E_INVALID),           # inner stride
    (dict(k=8), _lib.PRISM_E_INVALID),                             # misaligned base
    (dict(topk=0), _lib.PRISM_E_INVALID),
    (dict(topk=257), _lib.PRISM_E_INVALID),
    (dict(Sk=40000, ks=(40000 * 256, 40000 * 128, 128, 1), topk=20000), _lib.PRISM_E_UNSUPPORTED),
    (dict(mode=3), _lib.PRISM_E_INVALID),
    (dict(mode=1, topk=8), _lib.PRISM_E_INVALID),                 # blockmax: topk 1 or 4
    (dict(mode=1, topk=4, Sk=200, ks=(200 * 256, 200 * 128, 128, 1)), _lib.PRISM_E_INVALID),  # Sk % 128
    (dict(inv=16, pos=(1 << 22) - 10), _lib.PRISM_E_UNSUPPORTED),  # RoPE positions beyond 2^22
    (dict(base=-1), _lib.PRISM_E_INVALID),
    (dict(wsb=100), _lib.PRISM_E_WORKSPACE),
    (dict(ws=None), _lib.PRISM_E_WORKSPACE),
])
def test_argument_validation(lib, over, code):
    rc = _call(lib, **over)
    assert rc == code, (rc, _lib.last_error())
    assert _lib.last_error()


def test_rope_streaming_needs_the_planes(lib):
    # RoPE'd keys on the streaming path: the plain streaming workspace is refused
    # (before any CUDA call), naming the size function that covers the planes
    shape = dict(Hq=4, Hkv=2, Sq=64, Sk=256, qs=(64 * 4 * 128, 64 * 128, 128, 1), mode=_lib.MODE_EXACT_STREAM,
                 inv=16)
    plain = lib.prism_einsum_topk_workspace_size(1, 4, 64, 256, 8, _lib.MODE_EXACT_STREAM)
    rope = lib.prism_einsum_topk_rope_workspace_size(1, 4, 2, 64, 256, 8, _lib.MODE_EXACT_STREAM, _lib.RECALL_QK)
    assert rope == (plain + 255) // 256 * 256 + 2 * 256 * 512
    assert _call(lib, wsb=plain, **shape) == _lib.PRISM_E_WORKSPACE
    assert "prism_einsum_topk_rope_workspace_size" in _lib.last_error()


def test_merge_argument_validation(lib):
    rc = lib.prism_topk_merge(16, 16, 4, 10, 10, 3, 16, None, 16, 1 << 20, None)  # ld % 4 != 0
    assert rc == _lib.PRISM_E_INVALID
    rc = lib.prism_topk_merge(16, 16, 4, 12, 12, 13, 16, None, 16, 1 << 20, None)  # topk > n
    assert rc == _lib.PRISM_E_INVALID
    rc = lib.prism_topk_merge(16, 16, 4, 12, 12, 3, 16, None, 16, 8, None)  # workspace too small
    assert rc == _lib.PRISM_E_WORKSPACE


def test_error_maps_to_assertion():
    with pytest.raises(AssertionError):
        _lib.check(_lib.PRISM_E_INVALID, "x")
    with pytest.raises(pb.PrismLibraryError):
        _lib.check(_lib.PRISM_E_CUDA, "x")


def _call_weighted(lib, **over):
    args = dict(q=16, k=16, v=16, inv=None, dtype=0, B=1, Hq=4, Hkv=2, Sq=1, Sk=256, D=128, Dv=128,
                qs=(512, 128, 128, 1), ks=(65536, 32768, 128, 1), vs=(65536, 32768, 128, 1), pos=0,
                causal=-1, rw=_lib.RECALL_QKV2, topk=8, mode=0, base=0, oi=16, os=None, ws=256,
                wsb=1 << 20, stream=None)
    args.update(over)
    return lib.prism_einsum_topk_weighted(
        args["q"], args["k"], args["v"], args["inv"], args["dtype"], args["B"], args["Hq"], args["Hkv"],
        args["Sq"], args["Sk"], args["D"], args["Dv"], _lib.i64_array(args["qs"]),
        _lib.i64_array(args["ks"]), _lib.i64_array(args["vs"]), args["pos"], args["causal"], args["rw"],
        args["topk"], args["mode"], args["base"], args["oi"], args["os"], args["ws"], args["wsb"],
        args["stream"])


@pytest.mark.parametrize("over,code", [
    (dict(rw=3), _lib.PRISM_E_INVALID),                               # unknown weighting
    (dict(v=None), _lib.PRISM_E_INVALID),
    (dict(Dv=100, vs=(51200, 25600, 100, 1)), _lib.PRISM_E_UNSUPPORTED),  # Dv % 8
    (dict(vs=(65536, 32768, 128, 2)), _lib.PRISM_E_INVALID),          # inner stride
    (dict(v=8), _lib.PRISM_E_INVALID),                                # misaligned base
    (dict(vs=(65536, 32768, 132, 1)), _lib.PRISM_E_INVALID),          # key stride not 16-byte
    (dict(q=None), _lib.PRISM_E_INVALID),                             # shared checks still apply
    (dict(wsb=100), _lib.PRISM_E_WORKSPACE),
    (dict(rw=_lib.RECALL_QK, v=None, topk=0), _lib.PRISM_E_INVALID),  # qk ignores v
])
def test_weighted_argument_validation(lib, over, code):
    rc = _call_weighted(lib, **over)
    assert rc == code, (rc, _lib.last_error())
    assert _lib.last_error()


def test_recall_type_errors_match_reference():
    # the messages of ReAttentionMethod._apply_recall_weight (reattention.py:834-842)
    from prism_test_b200.kernels import _recall_weight_code
    assert _recall_weight_code("qk") == _lib.RECALL_QK
    assert _recall_weight_code("qkv") == _lib.RECALL_QKV
    assert _recall_weight_code("qkv2") == _lib.RECALL_QKV2
    with pytest.raises(ValueError, match="'_pe' variants are not implemented"):
        _recall_weight_code("qkv2_pe")
    with pytest.raises(ValueError, match="Use one of: qk, qkv, qkv2"):
        _recall_weight_code("k")


def test_rope_workspace_size(lib):
    # decode shapes (fewer than 128 query rows per KV head): the plain size
    plain = lib.prism_einsum_topk_weighted_workspace_size(1, 32, 8, 1, 131072, 4096, 0, _lib.RECALL_QK)
    assert lib.prism_einsum_topk_rope_workspace_size(1, 32, 8, 1, 131072, 4096, 0, _lib.RECALL_QK) == plain
    # prefill shapes: + the un-rotated hi / lo planes, B * Hkv * Sk * 512 bytes
    for args in ((2, 32, 8, 32, 9000, 512, 0, _lib.RECALL_QK),           # score matrix
                 (1, 32, 8, 4096, 131072, 2048, 0, _lib.RECALL_QK),      # streaming by itself
                 (1, 8, 2, 64, 20000, 300, _lib.MODE_EXACT_STREAM, _lib.RECALL_QK),
                 (1, 8, 2, 128, 8192, 1, _lib.MODE_BLOCKMAX, _lib.RECALL_QK),
                 (1, 8, 2, 64, 5000, 100, 0, _lib.RECALL_QKV2)):
        base = lib.prism_einsum_topk_weighted_workspace_size(*args)
        B, Hkv, Sk = args[0], args[2], args[4]
        want = (base + 255) // 256 * 256 + B * Hkv * Sk * 512
        assert lib.prism_einsum_topk_rope_workspace_size(*args) == want, args
    assert lib.prism_einsum_topk_rope_workspace_size(1, 8, 3, 64, 5000, 100, 0, 0) == \
        lib.prism_einsum_topk_weighted_workspace_size(1, 8, 3, 64, 5000, 100, 0, 0)
    assert lib.prism_einsum_topk_rope_workspace_size(0, 8, 2, 64, 5000, 100, 0, 0) == 0


def test_weighted_workspace_size(lib):
    base = lib.prism_einsum_topk_workspace_size(1, 32, 1, 131072, 4096, 0)
    assert lib.prism_einsum_topk_weighted_workspace_size(1, 32, 8, 1, 131072, 4096, 0, _lib.RECALL_QK) == base
    # weights [B * Hkv, Sk rounded to 4] fp32 after the 256-byte aligned base
    want = (base + 255) // 256 * 256 + 8 * 131072 * 4
    assert lib.prism_einsum_topk_weighted_workspace_size(1, 32, 8, 1, 131072, 4096, 0, _lib.RECALL_QKV2) == want
    odd = lib.prism_einsum_topk_workspace_size(1, 4, 5, 1001, 3, 0)
    got = lib.prism_einsum_topk_weighted_workspace_size(1, 4, 2, 5, 1001, 3, 0, _lib.RECALL_QKV)
    assert got == (odd + 255) // 256 * 256 + (2 * 1004 * 4 + 255) // 256 * 256
    assert lib.prism_einsum_topk_weighted_workspace_size(1, 4, 2, 5, 1001, 3, 0, 9) == 0


def test_peer_exchange_validation(lib):
    # argument checks of the peer exchange entry points run before any CUDA call
    assert lib.prism_peer_buffer_bytes(32, 8192) == _lib.PEER_HEADER_BYTES + 32 * 8192 * 8
    assert lib.prism_peer_buffer_bytes(0, 8) == 0
    fake = (ctypes.c_void_p * 3)(1 << 20, 2 << 20, 3 << 20)  # never dereferenced
    assert lib.prism_peer_publish(fake, 0, 0, None) == _lib.PRISM_E_UNSUPPORTED
    assert lib.prism_peer_publish(fake, _lib.PEER_MAX_RANKS + 1, 0, None) == _lib.PRISM_E_UNSUPPORTED
    assert lib.prism_peer_publish(fake, 3, 3, None) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_publish(None, 3, 0, None) == _lib.PRISM_E_INVALID
    mis = (ctypes.c_void_p * 2)(1 << 20, (2 << 20) + 8)
    assert lib.prism_peer_publish(mis, 2, 0, None) == _lib.PRISM_E_INVALID
    nul = (ctypes.c_void_p * 2)(1 << 20, None)
    assert lib.prism_peer_publish(nul, 2, 0, None) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_wait_acks(fake, 0, 0, 0, None) == _lib.PRISM_E_UNSUPPORTED
    assert lib.prism_peer_wait_acks(fake, 3, 5, 0, None) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_wait_acks(mis, 2, 0, 0, None) == _lib.PRISM_E_INVALID
    out = 4 << 20
    assert lib.prism_peer_merge(fake, 3, 0, 4, 16, 1, 0, None, None, None) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_merge(fake, 3, 0, 0, 16, 1, 0, out, None, None) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_merge(fake, 3, 0, 4, 16385, 1, 0, out, None, None) == _lib.PRISM_E_UNSUPPORTED
    h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    assert lib.prism_peer_alloc(1 << 20, None, h) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_alloc(100, ctypes.byref(ctypes.c_void_p()), h) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_open(None, ctypes.byref(ctypes.c_void_p())) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_close(None) == _lib.PRISM_E_INVALID
    assert lib.prism_peer_free(None) == _lib.PRISM_E_INVALID
