"""The Node-API addon (hachiue_b200/napi/hachiue_napi.c), compiled with gcc
against a declared subset of Node-API (tests/napi_mock/node_api.h) and run on
a mock of the Node-API runtime (tests/napi_mock/mock_napi.c), so that its
exports are called the way the reference's engine would call them from JS
(src/engine.ts:1056-1075: dispatch(shader, uniform words, storage buffers)).

CPU: registration, the version, and the argument checks that run before any
device call.  GPU: the engine's Q8 sequence (kv_append_q8 x2, attention_q8)
through the addon with host buffers, bit-exact cache and oracle-checked
output, in both Q8_0 conventions, plus the errors a JS caller sees."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MOCK = os.path.join(ROOT, "tests", "napi_mock")
SHIM = os.path.join(ROOT, "hachiue_b200", "napi", "hachiue_napi.c")
GOLDEN = os.path.join(ROOT, "tests", "golden")

EXPORTS = {"version", "create", "destroy", "alloc", "free", "copyToDevice", "copyToHost", "sync", "dispatch",
           "setQ8Convention", "setOption", "deviceStatus"}

# napi_typedarray_type of each numpy dtype
_TA = {np.dtype(np.int8): 0, np.dtype(np.uint8): 1, np.dtype(np.int16): 3, np.dtype(np.uint16): 4,
       np.dtype(np.int32): 5, np.dtype(np.uint32): 6, np.dtype(np.float32): 7, np.dtype(np.float64): 8,
       np.dtype(np.int64): 9, np.dtype(np.uint64): 10}


class JSError(Exception):
    pass


class Big(int):
    """A JS bigint argument."""


class Foreign:
    """An External made by some other addon."""

    def __init__(self, p):
        self.p = p


class Value:
    """An opaque JS value returned by the addon (a handle)."""

    def __init__(self, v):
        self.v = v


class Addon:
    """The addon loaded into one mock Node-API environment."""

    def __init__(self, path):
        lib = self.lib = ctypes.CDLL(path)
        vp = ctypes.c_void_p
        for name, res, args in (("mock_env_new", vp, []), ("mock_env_free", None, [vp]), ("mock_register", ctypes.c_int, [vp]),
                                ("mock_export_name", ctypes.c_char_p, [vp, ctypes.c_int]), ("mock_gc", ctypes.c_int, [vp]),
                                ("mock_undefined", vp, [vp]), ("mock_number", vp, [vp, ctypes.c_double]),
                                ("mock_bool", vp, [vp, ctypes.c_int]), ("mock_string", vp, [vp, ctypes.c_char_p]),
                                ("mock_bigint", vp, [vp, ctypes.c_uint64, ctypes.c_int]),
                                ("mock_typedarray", vp, [vp, ctypes.c_int, vp, ctypes.c_size_t]),
                                ("mock_foreign_external", vp, [vp, vp]),
                                ("mock_call", vp, [vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(vp)]),
                                ("mock_take_exception", ctypes.c_char_p, [vp]), ("mock_kind", ctypes.c_int, [vp]),
                                ("mock_as_number", ctypes.c_double, [vp]), ("mock_as_bigint", ctypes.c_uint64, [vp])):
            f = getattr(lib, name)
            f.restype, f.argtypes = res, args
        self.env = lib.mock_env_new()
        self.n_exports = lib.mock_register(self.env)
        self.keep = []

    def exports(self):
        return {self.lib.mock_export_name(self.env, i).decode() for i in range(self.n_exports)}

    def _js(self, x):
        L, e = self.lib, self.env
        if x is None:
            return L.mock_undefined(e)
        if isinstance(x, Value):
            return x.v
        if isinstance(x, Foreign):
            return L.mock_foreign_external(e, x.p)
        if isinstance(x, bool):
            return L.mock_bool(e, int(x))
        if isinstance(x, Big):
            return L.mock_bigint(e, int(x) & (2**64 - 1), int(0 <= x < 2**64))
        if isinstance(x, (int, float)):
            return L.mock_number(e, float(x))
        if isinstance(x, str):
            return L.mock_string(e, x.encode())
        if isinstance(x, np.ndarray):
            assert x.flags.c_contiguous
            self.keep.append(x)
            return L.mock_typedarray(e, _TA[x.dtype], x.ctypes.data, x.size)
        raise TypeError(type(x))

    def __call__(self, name, *args):
        argv = (ctypes.c_void_p * max(1, len(args)))(*[self._js(a) for a in args])
        r = self.lib.mock_call(self.env, name.encode(), len(args), argv)
        exc = self.lib.mock_take_exception(self.env)
        if exc is not None:
            raise JSError(exc.decode())
        assert r, f"no export {name}"
        kind = self.lib.mock_kind(r)
        if kind == 0:
            return None
        if kind == 1:
            return self.lib.mock_as_number(r)
        if kind == 4:
            return Big(self.lib.mock_as_bigint(r))
        return Value(r)

    def gc(self):
        return self.lib.mock_gc(self.env)

    def close(self):
        self.lib.mock_env_free(self.env)


@pytest.fixture(scope="module")
def addon_path(tmp_path_factory):
    from hachiue_b200 import _lib, build
    build.build()
    libdir = os.path.dirname(_lib.LIB_PATH)
    out = str(tmp_path_factory.mktemp("napi") / "hachiue_cuda_mock.so")
    subprocess.run(["gcc", "-shared", "-fPIC", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror",
                    "-DNODE_GYP_MODULE_NAME=hachiue_cuda", "-I", MOCK, "-I", os.path.join(ROOT, "include"),
                    SHIM, os.path.join(MOCK, "mock_napi.c"), "-L", libdir, "-lhachiue_cuda",
                    f"-Wl,-rpath,{libdir}", "-o", out], check=True)
    return out


@pytest.fixture
def node(addon_path):
    a = Addon(addon_path)
    yield a
    a.close()


def test_addon_registers_every_export(node):
    assert node.exports() == EXPORTS


def test_version_is_the_abi_version(node):
    assert node("version") == 3


def test_arguments_are_checked_before_any_device_call(node):
    words = np.zeros(8, np.uint32)
    bufs = np.zeros(6, np.uint64)
    with pytest.raises(JSError, match="^hachiue: too few arguments$"):
        node("dispatch")
    with pytest.raises(JSError, match="^hachiue: expected a handle from create\\(\\)$"):
        node("dispatch", 1, "attention_q8", words, bufs)
    with pytest.raises(JSError, match="^hachiue: expected a handle from create\\(\\)$"):
        node("dispatch", Foreign(ctypes.addressof(ctypes.c_uint64(0x68637531))), "attention_q8", words, bufs)
    with pytest.raises(JSError, match="^hachiue: expected a handle from create\\(\\)$"):
        node("sync", Foreign(None))
    with pytest.raises(JSError, match="^hachiue: a size must not be negative$"):
        node("create", 0, -1)
    with pytest.raises(JSError, match="^hachiue: expected a number$"):
        node("create", "0", 0)
    assert node.gc() == 0


def test_create_without_gpu_throws_the_library_message(node):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(JSError, match="^hachiue: hcu_create"):
        node("create", 0, 0)
    assert node.gc() == 0  # nothing was wrapped


def _golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def _engine_sequence(node, h, d, q8_format):
    """forwardSegment's dispatches (src/engine.ts:1305-1317) through the addon:
    kv_append_q8 for K and V per segment, then attention_q8; every buffer a
    device pointer from alloc(), inputs and results copied with host arrays."""
    S, H, KV, Dh, pos, W = (int(x) for x in d["meta"])
    rows, nb = pos + S, Dh // 32
    node("setQ8Convention", h, q8_format)
    q, k, v = (np.ascontiguousarray(d[n], np.float32) for n in ("q", "k", "v"))
    ptr = {}
    for n, nbytes in (("q", q.nbytes), ("k", k.nbytes), ("v", v.nbytes), ("kq", rows * KV * Dh), ("vq", rows * KV * Dh),
                      ("ks", rows * KV * nb * 4), ("vs", rows * KV * nb * 4), ("out", S * H * Dh * 4)):
        ptr[n] = node("alloc", h, nbytes)
    for n, x in (("q", q), ("k", k), ("v", v)):
        node("copyToDevice", h, ptr[n], x)
    zero8 = np.zeros(rows * KV * Dh, np.int8)
    zerof = np.zeros(rows * KV * nb, np.float32)
    for n, x in (("kq", zero8), ("vq", zero8), ("ks", zerof), ("vs", zerof)):
        node("copyToDevice", h, ptr[n], x)
    row_bytes = KV * Dh * 4
    for lo, hi in ((0, pos), (pos, rows)):
        if hi > lo:
            for src, q8, sc in (("k", "kq", "ks"), ("v", "vq", "vs")):
                words = np.array([hi - lo, KV, Dh, lo, 0, 0, 0, 0], np.uint32)
                bufs = np.array([int(ptr[src]) + lo * row_bytes, int(ptr[q8]), int(ptr[sc])], np.uint64)
                node("dispatch", h, "kv_append_q8", words, bufs)
    words = np.array([S, H, KV, Dh, pos, W, 0, 0], np.uint32)
    bufs = np.array([int(ptr[n]) for n in ("q", "kq", "ks", "vq", "vs", "out")], np.uint64)
    node("dispatch", h, "attention_q8", words, bufs)
    node("sync", h)
    got = {"kq": np.zeros((rows, KV, Dh), np.int8), "vq": np.zeros((rows, KV, Dh), np.int8),
           "ks": np.zeros((rows, KV, nb), np.float32), "vs": np.zeros((rows, KV, nb), np.float32),
           "out": np.zeros((S, H, Dh), np.float32)}
    for n, x in got.items():
        node("copyToHost", h, x, ptr[n])
    for p in ptr.values():
        node("free", h, p)
    return got


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["attn_q8_decode", "attn_q8_segment"])
def test_engine_q8_sequence_through_the_addon(node, name):
    import oracle
    from tests.conftest import rel_l2
    d = _golden(name)
    h = node("create", 0, 0)
    got = _engine_sequence(node, h, d, 3)  # HCU_KV_Q8_0, the JS backend's convention
    for n in ("kq", "ks", "vq", "vs"):
        np.testing.assert_array_equal(got[n], d[n])
    assert rel_l2(got["out"], d["out"]) < 1e-4
    assert node("deviceStatus", h, False) == 0

    # the WGSL ops' convention (scale = amax), checked against its restatement
    S, H, KV, Dh, pos, W = (int(x) for x in d["meta"])
    rows, nb = pos + S, Dh // 32
    got = _engine_sequence(node, h, d, 4)  # HCU_KV_Q8_0_WGSL
    kq, vq = np.zeros((rows, KV, Dh), np.int8), np.zeros((rows, KV, Dh), np.int8)
    ka, va = np.zeros((rows, KV, nb), np.float32), np.zeros((rows, KV, nb), np.float32)
    for lo, hi in ((0, pos), (pos, rows)):
        if hi > lo:
            oracle.append_kv_q8_wgsl(np.ascontiguousarray(d["k"][lo:hi]), kq, ka, lo)
            oracle.append_kv_q8_wgsl(np.ascontiguousarray(d["v"][lo:hi]), vq, va, lo)
    for n, ref in (("kq", kq), ("ks", ka), ("vq", vq), ("vs", va)):
        np.testing.assert_array_equal(got[n], ref)
    assert rel_l2(got["out"], oracle.attention_q8_wgsl(d["q"], kq, ka, vq, va, pos, W)) < 1e-4
    node("destroy", h)
    assert node.gc() == 1


@pytest.mark.gpu
def test_errors_a_js_caller_sees(node):
    h = node("create", 0, 0)
    words = np.zeros(8, np.uint32)
    with pytest.raises(JSError, match="^hachiue: missing pipeline gemv_q4_k$"):
        node("dispatch", h, "gemv_q4_k", words, np.zeros(1, np.uint64))
    with pytest.raises(JSError, match="expected 6 storage buffers"):
        node("dispatch", h, "attention_q8", np.array([1, 16, 8, 128, 0, 0, 0, 0], np.uint32), np.zeros(2, np.uint64))
    with pytest.raises(JSError, match="^hachiue: uniform words must be a Uint32Array\\(8\\)$"):
        node("dispatch", h, "attention_q8", np.zeros(4, np.uint32), np.zeros(6, np.uint64))
    with pytest.raises(JSError, match="^hachiue: buffers must be a BigUint64Array of device pointers$"):
        node("dispatch", h, "attention_q8", words, np.zeros(6, np.float64))
    with pytest.raises(JSError, match="^hachiue: shader name too long$"):
        node("dispatch", h, "x" * 80, words, np.zeros(1, np.uint64))
    with pytest.raises(JSError, match="^hachiue: expected a device pointer \\(bigint\\)$"):
        node("free", h, Big(-1))
    with pytest.raises(JSError, match="^hachiue: hcu_set_q8_convention"):
        node("setQ8Convention", h, 7)
    assert node("deviceStatus", h, True) == 0
    node("destroy", h)
    with pytest.raises(JSError, match="^hachiue: the handle was destroyed$"):
        node("sync", h)
    with pytest.raises(JSError, match="^hachiue: the handle was destroyed$"):
        node("destroy", h)
    assert node.gc() == 1  # frees the wrapper; the context is not destroyed twice


@pytest.mark.gpu
def test_collected_handle_releases_its_context(node):
    h = node("create", 0, 0)
    p = node("alloc", h, 1 << 20)
    node("free", h, p)
    assert node.gc() == 1  # hcu_destroy from the finalizer
    assert node.gc() == 0
