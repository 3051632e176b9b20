"""C-ABI and host logic of libtb_b200.so, on the CPU (no device work).

- the library loads and exports every function declared in include/*.h;
- ABI struct layouts (TbTensor as the engine lays it out, tensor.h:47-54);
- the device-aware registry: routing by priority and by device, with the
  reference's own CPU adapters (oracle/_ref) registered as "cpu", and the
  engine's dispatch packing;
- the b200 backend rejects host tensors before touching a device;
- row partitioning and the sharded-embedding exchange plan.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("tb_b200.h", "tb_backend.h", "tb_types.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(tb_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def exported_functions():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", T.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_library_loads_and_reports_version():
    assert T.lib().tb_b200_version() == 1


# Declared for the engine (tb_backend.h replaces its backend.h) but defined
# by the engine itself, not by this library.
ENGINE_DEFINED = {"tb_backend_cpu_init"}


def test_every_declared_function_is_exported():
    decl = declared_functions() - ENGINE_DEFINED
    assert len(decl) > 60
    missing = decl - exported_functions()
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # and the Python binding knows every one of them
    assert decl <= set(T.SIGNATURES), sorted(decl - set(T.SIGNATURES))


def test_abi_struct_layouts():
    assert C.sizeof(T.TbTensor) == 88
    assert T.TbTensor.rank.offset == 72 and T.TbTensor.dtype.offset == 76
    assert T.TbTensor.device.offset == 80 and T.TbTensor.owns_data.offset == 84
    assert C.sizeof(T.LayerChain) == 160


def test_no_device_is_not_an_error():
    n = C.c_int(-1)
    assert T.lib().tb_b200_device_count(C.byref(n)) == 0
    assert n.value >= 0


def test_decoder_entry_points_check_arguments_before_device_work():
    """The decoder's entry points reject bad arguments before they touch a
    device (so these run without a GPU): TB_ERR_INVALID_ARG (8) and
    TB_ERR_INVALID_SHAPE (9)."""
    L = T.lib()
    h = C.c_void_p()
    assert L.tb_b200_runner_create(None, C.byref(h)) == 8
    d = T.RunnerDesc()  # hidden 0
    assert L.tb_b200_runner_create(C.byref(d), C.byref(h)) == 9 and not h.value
    assert L.tb_b200_runner_forward(None, 0, None) == 8
    assert L.tb_b200_runner_logits(None, None) == 8
    assert L.tb_b200_runner_reset(None) == 8
    assert L.tb_b200_runner_destroy(None) == 0
    buf = (C.c_float * 64)()
    p = C.cast(buf, C.c_void_p)
    args = [p] * 7 + [None]
    assert L.tb_b200_decode_attention(7, 8, 8, 64, 16, *args) == 8     # no such layout
    assert L.tb_b200_decode_attention(0, 8, 8, 512, 16, *args) == 9    # head_dim > 256
    assert L.tb_b200_decode_attention(0, 8, 3, 64, 16, *args) == 9     # heads not a multiple
    assert L.tb_b200_decode_attention(1, 8, 8, 64, 16, None, *args[1:]) == 8
    assert L.tb_b200_sparse24_linear(4, 12, p, p, p, None, p, None) == 9  # 3 groups: no pairs
    assert L.tb_b200_sparse24_linear(4, 16, None, p, p, None, p, None) == 8
    assert L.tb_b200_sparse24_linear(-1, 16, p, p, p, None, p, None) == 9
    assert L.tb_b200_sparse24_pack(4, 16, None, p, p, p, p, None) == 8


def test_p2p_entry_points_check_arguments_before_device_work():
    """The peer-memory gather and its IPC set-up reject bad arguments before
    any CUDA call: TB_ERR_INVALID_ARG (8), TB_ERR_INVALID_SHAPE (9),
    TB_ERR_UNSUPPORTED_DTYPE (10)."""
    L = T.lib()
    buf = (C.c_float * 64)()
    p = C.cast(buf, C.c_void_p)
    shards = (C.c_void_p * 8)(*([p.value] * 8))
    off, out = C.c_int64(), C.c_void_p()
    assert L.tb_b200_p2p_export(None, p, C.byref(off)) == 8
    assert L.tb_b200_p2p_export(p, None, C.byref(off)) == 8
    assert L.tb_b200_p2p_import(None, 0, C.byref(out)) == 8
    assert L.tb_b200_p2p_import(p, -1, C.byref(out)) == 8
    assert L.tb_b200_p2p_close(None, 0) == 8
    assert L.tb_b200_p2p_close(p, -16) == 8
    f = L.tb_b200_embedding_sharded_p2p
    assert f(0, -1, 16, 100, p, shards, 2, p, None) == 9
    assert f(4, 8, 16, 100, p, shards, 2, p, None) == 10     # int32 rows: not a table type
    assert f(0, 8, 16, 100, p, shards, 0, p, None) == 8      # no ranks
    assert f(0, 8, 16, 100, p, shards, 9, p, None) == 8      # more than 8 ranks
    assert f(0, 8, 16, 1, p, shards, 2, p, None) == 8        # fewer rows than ranks
    assert f(0, 8, 16, 100, None, shards, 2, p, None) == 8
    assert f(0, 8, 16, 100, p, None, 2, p, None) == 8
    assert f(0, 8, 16, 100, p, shards, 2, None, None) == 8
    shards[1] = None
    assert f(0, 8, 16, 100, p, shards, 2, p, None) == 8      # a missing shard
    assert f(0, 0, 16, 100, None, None, 2, None, None) == 0  # no tokens: nothing to do


def test_empty_inputs_are_no_ops():
    """Zero rows (or zero elements) is nothing to do: every row op returns
    TB_OK before it looks for a device or touches a pointer, as the
    reference's loops do nothing for n = 0."""
    L = T.lib()
    N, F = None, C.c_float
    assert L.tb_b200_softmax(T.F32, 0, 10, N, N, N, N) == 0
    assert L.tb_b200_softmax(T.BF16, 5, 0, N, N, N, N) == 0
    assert L.tb_b200_argmax(T.F32, 0, 10, N, N, N) == 0
    assert L.tb_b200_silu(T.F32, 0, N, N, N) == 0
    assert L.tb_b200_gelu(T.BF16, 0, N, N, N) == 0
    assert L.tb_b200_swiglu(T.F32, 0, N, N, N, N) == 0
    assert L.tb_b200_residual_add(T.F32, 0, N, N, N, N) == 0
    assert L.tb_b200_rms_norm(T.F32, 0, 4, N, N, N, F(1e-5), N) == 0
    assert L.tb_b200_residual_rms_norm(T.BF16, 0, 4, N, N, N, N, N, F(1e-5), N) == 0
    assert L.tb_b200_embedding(T.F32, 0, 16, 100, N, N, N, N) == 0
    assert L.tb_b200_rope_rows(T.F32, 0, 4, 4, 64, N, N, N, F(1e4), N, 0, N) == 0


def test_partition_rule():
    lo, hi = C.c_int64(), C.c_int64()
    for total, parts in [(16384, 8), (10, 3), (5, 8), (128256, 7)]:
        spans = []
        for p in range(parts):
            assert T.lib().tb_b200_partition(total, parts, p, C.byref(lo), C.byref(hi)) == 0
            spans.append((lo.value, hi.value))
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(spans[i][1] == spans[i + 1][0] for i in range(parts - 1))
        sizes = [h - l for l, h in spans]
        assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)


def shard_plan(ids, vocab, nranks, rank):
    n = len(ids)
    sc = np.zeros(nranks, np.int64)
    rc = np.zeros(nranks, np.int64)
    bufs = [np.zeros(n + 1, np.int32) for _ in range(4)]
    nl = C.c_int64()
    ids = np.ascontiguousarray(ids, np.int32)
    code = T.lib().tb_b200_shard_plan(n, vocab, nranks, rank, ids.ctypes.data, sc.ctypes.data,
                                      rc.ctypes.data, *[b.ctypes.data for b in bufs], C.byref(nl))
    assert code == 0
    s, r, ld, ls = bufs
    return sc, rc, s[:sc.sum()], r[:rc.sum()], ld[:nl.value], ls[:nl.value]


def bounds(total, parts):
    base, extra = divmod(total, parts)
    lo = [p * base + min(p, extra) for p in range(parts)]
    return [(l, l + base + (1 if p < extra else 0)) for p, l in enumerate(lo)]


@pytest.mark.parametrize("n,vocab,nranks", [(64, 100, 2), (1000, 128256, 8), (7, 10, 3),
                                            (0, 16, 4)])
def test_shard_plan_reassembles_the_gather(n, vocab, nranks):
    """Simulate every rank's plan and exchange in numpy; the result must be the
    full-table gather (tb_cpu_embedding_f32, src/ops/embedding.c:4-14)."""
    rng = np.random.default_rng(n + vocab)
    ids = rng.integers(0, vocab, n).astype(np.int32)
    table = rng.standard_normal((vocab, 4), dtype=np.float32)
    vb, tb = bounds(vocab, nranks), bounds(n, nranks)
    plans = [shard_plan(ids, vocab, nranks, r) for r in range(nranks)]
    for me in range(nranks):
        tlo, thi = tb[me]
        out = np.full((thi - tlo, 4), np.nan, np.float32)
        sc, rc, send, recv, ld, ls = plans[me]
        shard = table[vb[me][0]:vb[me][1]]
        out[ld] = shard[ls]
        ro = 0
        for src in range(nranks):
            if src == me:
                continue
            ssc, _, ssend, _, _, _ = plans[src]
            off = int(ssc[:me].sum())
            rows = table[vb[src][0]:vb[src][1]][ssend[off:off + ssc[me]]]
            assert rc[src] == ssc[me]
            out[recv[ro:ro + rc[src]]] = rows
            ro += rc[src]
        np.testing.assert_array_equal(out, O.embedding(ids[tlo:thi], table))


def test_shard_plan_rejects_out_of_range_ids():
    z = np.zeros(8, np.int64)
    b = np.zeros(8, np.int32)
    nl = C.c_int64()
    ids = np.array([3, 100], np.int32)
    assert T.lib().tb_b200_shard_plan(2, 100, 2, 0, ids.ctypes.data, z.ctypes.data, z.ctypes.data,
                                      b.ctypes.data, b.ctypes.data, b.ctypes.data, b.ctypes.data,
                                      C.byref(nl)) == 8


# ------------------------------------------------------------- registry
OpFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_void_p), C.c_int, C.c_void_p)


class Backend(C.Structure):
    _fields_ = [("name", C.c_char_p), ("priority", C.c_int), ("ops", C.c_void_p * T.OP["COUNT"])]


_alive = []  # the registry copies the vtable, not the name string it points to


def make_backend(name, prio, slots):
    be = Backend()
    _alive.append(be)
    be.name = name.encode()
    be.priority = prio
    for op, fn in slots.items():
        be.ops[T.OP[op]] = C.cast(fn, C.c_void_p)
    return be


@pytest.fixture
def registry():
    L = T.lib()
    L.tb_backend_reset()
    yield L
    L.tb_backend_reset()


def test_registry_priority_and_device_routing(registry):
    calls = []
    fns = {n: OpFn(lambda o, i, n_, p, n=n: calls.append(n) or 0) for n in ("lo", "hi", "dev")}
    registry.tb_backend_register(C.byref(make_backend("lo", 0, {"GELU": fns["lo"]})))
    registry.tb_backend_register(C.byref(make_backend("hi", 50, {"GELU": fns["hi"]})))
    registry.tb_backend_register_device(C.byref(make_backend("dev", 200, {"GELU": fns["dev"]})),
                                        T.DEVICE_CUDA)
    assert registry.tb_backend_count() == 3
    best = C.cast(registry.tb_backend_get_best(T.OP["GELU"]), C.POINTER(Backend)).contents
    assert best.name == b"dev"  # the engine's get_best is device-blind
    host = T.TbTensor(device=T.DEVICE_CPU)
    dev = T.TbTensor(device=T.DEVICE_CUDA)
    assert registry.tb_dispatch_gelu(C.byref(host), C.byref(host)) == 0
    assert registry.tb_dispatch_gelu(C.byref(dev), C.byref(dev)) == 0
    assert calls == ["hi", "dev"]
    # no backend has a slot: TB_ERR_BACKEND_NOT_FOUND (src/backend/cpu/registry.c:93)
    assert registry.tb_dispatch_silu(C.byref(host), C.byref(host)) == 14
    assert not registry.tb_backend_get_best(T.OP["COUNT"])


def test_registry_capacity_is_eight(registry):
    be = make_backend("x", 1, {})
    for _ in range(8):
        assert registry.tb_backend_register(C.byref(be)) == 0
    assert registry.tb_backend_register(C.byref(be)) == -1


def test_dispatch_packs_inputs_like_the_engine(registry):
    seen = {}

    def fn(out, inputs, n, params):
        seen["n"] = n
        seen["inputs"] = [inputs[i] for i in range(n)]
        seen["eps"] = C.cast(params, C.POINTER(C.c_float))[0]
        return 0

    cb = OpFn(fn)
    registry.tb_backend_register(C.byref(make_backend("spy", 0, {"RMS_NORM": cb})))
    y, x, w = T.TbTensor(), T.TbTensor(), T.TbTensor()
    assert registry.tb_dispatch_rms_norm(C.byref(y), C.byref(x), C.byref(w), C.c_float(0.25)) == 0
    assert seen["n"] == 2 and seen["eps"] == 0.25
    assert seen["inputs"] == [C.addressof(x), C.addressof(w)]


def test_b200_backend_registers_for_cuda_and_rejects_host_tensors(registry):
    assert registry.tb_backend_b200_init() == 0
    assert registry.tb_backend_b200_init() == 0  # idempotent
    assert registry.tb_backend_count() == 1
    be = C.cast(registry.tb_backend_get(0), C.POINTER(Backend)).contents
    assert be.name == b"b200" and be.priority == 200
    filled = {op for op, v in T.OP.items() if op != "COUNT" and be.ops[v]}
    assert filled == {"RMS_NORM", "RESIDUAL_ADD", "GELU", "SILU", "SOFTMAX", "ROPE", "EMBEDDING",
                      "RESIDUAL_RMS_NORM", "SWIGLU", "ARGMAX", "ROPE_ROWS", "LAYER_CHAIN",
                      "SPARSE_LINEAR", "DENSE_LINEAR"}
    a = np.zeros(16, np.float32)
    host = T.TbTensor(data=a.ctypes.data, rank=1, dtype=T.F32, device=T.DEVICE_CPU)
    host.shape[0] = 16
    # routing: nothing serves host tensors here
    assert registry.tb_dispatch_silu(C.byref(host), C.byref(host)) == 14
    # the op itself refuses host memory: no CPU fallback inside the backend
    fn = C.cast(be.ops[T.OP["SILU"]], OpFn)
    arr = (C.c_void_p * 1)(C.addressof(host))
    assert fn(C.addressof(host), arr, 1, None) == 8


def _ref_cpu_backend():
    """The reference's CPU adapters (src/backend/cpu/*.c, built into
    oracle/_ref) as a "cpu" TbBackend -- test infrastructure."""
    ref = C.CDLL(O.REF_SO)
    slots = {}
    for op, sym in [("RMS_NORM", "tb_cpu_rms_norm_dispatch"), ("GELU", "tb_cpu_gelu_dispatch"),
                    ("SILU", "tb_cpu_silu_dispatch"), ("SOFTMAX", "tb_cpu_softmax_dispatch"),
                    ("ROPE", "tb_cpu_rope_dispatch"),
                    ("RESIDUAL_ADD", "tb_cpu_residual_add_dispatch"),
                    ("EMBEDDING", "tb_cpu_embedding_dispatch")]:
        slots[op] = C.cast(getattr(ref, sym), OpFn)
    return ref, slots


@pytest.mark.skipif(not os.path.exists(O.REF_SO), reason="oracle/_ref not built here")
def test_host_tensors_reach_the_reference_cpu_backend(registry):
    ref, slots = _ref_cpu_backend()
    registry.tb_backend_register(C.byref(make_backend("cpu", 0, slots)))
    assert registry.tb_backend_b200_init() == 0
    rng = np.random.default_rng(3)
    x = rng.standard_normal(256).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    y = np.zeros_like(x)

    def tt(a):
        t = T.TbTensor(data=a.ctypes.data, rank=1, dtype=T.F32, device=T.DEVICE_CPU)
        t.shape[0] = a.size
        return t

    ty, tx, tw = tt(y), tt(x), tt(w)
    assert registry.tb_dispatch_rms_norm(C.byref(ty), C.byref(tx), C.byref(tw),
                                         C.c_float(1e-5)) == 0
    np.testing.assert_array_equal(y, O.rms_norm_vec(x, w, 1e-5))


def test_library_before_torch_keeps_torch_importable():
    """The library resolves NCCL at run time: loading it before torch must not
    claim the libnccl.so.2 soname with a different NCCL than torch's."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r); import tb_b200; tb_b200.lib(); import torch; "
            "print(torch.__version__)" % os.path.join(ROOT, "tensorbit-run_b200"))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]


PIN_REGISTRY_SO = os.path.join(ROOT, "oracle", "_ref", "libpinregistry.so")


@pytest.mark.skipif(not os.path.exists(PIN_REGISTRY_SO), reason="oracle/_ref not built here")
def test_engine_backend_registry_builds_against_the_b200_header():
    """The engine's own C++ registry (BackendRegistry, backend.hpp:19-53,
    unmodified) compiled with include/tb_backend.h in place of backend.h and
    its accelerator branch bound to tb_backend_b200_init, linked to
    libtb_b200.so (oracle/_ref/libpinregistry.so).  Its init registers "cpu"
    and "b200"; device-aware routing picks "b200" for CUDA tensors and
    "cpu" for host tensors; the engine's C++ rms_norm wrapper on host
    tensors reaches the reference's CPU kernel.  The engine's CPU adapters
    are compiled against the swapped header too, and the five added ops
    reach the CPU backend's compositions (tensorbit-run_b200/engine/
    cpu_rowops.c) for host tensors, bit-exact with the oracle over the
    reference's kernels.  In a fresh process: the registry is a process-wide
    singleton."""
    import subprocess
    import sys
    code = r'''
import ctypes as C, sys
import numpy as np
sys.path[:0] = sys.argv[2:4]
import tb_b200 as T
from oracle import oracle as O
L = C.CDLL(sys.argv[1])
L.pin_registry_best.restype = C.c_char_p
L.pin_registry_has.argtypes = [C.c_char_p]
L.pin_registry_rms_norm_host.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_float]
V, Z, F = C.c_void_p, C.c_size_t, C.c_float
L.pin_registry_residual_rms_norm_host.argtypes = [V] * 5 + [Z, Z, F]
L.pin_registry_swiglu_host.argtypes = [V] * 3 + [Z, Z]
L.pin_registry_argmax_host.argtypes = [V] * 2 + [Z, Z]
L.pin_registry_rope_rows_host.argtypes = [V] * 3 + [Z] * 4 + [F]
L.pin_registry_layer_chain_host.argtypes = [V] * 11 + [Z] * 6 + [F, F]
assert L.pin_registry_init() == 2
assert L.pin_registry_init() == 2  # init is once per process
assert L.pin_registry_has(b"cpu") and L.pin_registry_has(b"b200")
for op in ("RMS_NORM", "RESIDUAL_ADD", "GELU", "SILU", "SOFTMAX", "ROPE", "EMBEDDING"):
    assert L.pin_registry_best(T.OP[op], 1) == b"b200", op
    assert L.pin_registry_best(T.OP[op], 0) == b"cpu", op
for op in ("RESIDUAL_RMS_NORM", "SWIGLU", "ARGMAX", "ROPE_ROWS", "LAYER_CHAIN"):
    assert L.pin_registry_best(T.OP[op], 1) == b"b200", op
    assert L.pin_registry_best(T.OP[op], 0) == b"cpu", op  # engine/cpu_rowops.c
assert L.pin_registry_best(T.OP["LAYER_NORM"], 1) == b"cpu"  # no b200 slot: the cpu one
rng = np.random.default_rng(9)
x = rng.standard_normal(4096).astype(np.float32)
w = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float32)
y = np.zeros_like(x)
assert L.pin_registry_rms_norm_host(y.ctypes.data, x.ctypes.data, w.ctypes.data, x.size, 1e-5) == 0
assert np.array_equal(y, O.rms_norm_vec(x, w, 1e-5))
# the added ops on host tensors reach the CPU compositions of the engine's
# kernels: bit-exact with the oracle over the reference's own kernels
R, H, I, HQ, HKV, D = 6, 256, 704, 4, 2, 64
f = lambda *sh: rng.standard_normal(sh).astype(np.float32)
P = lambda a: a.ctypes.data
x2, r2, g2, u2 = f(R, H), f(R, H), f(R, I), f(R, I)
w2 = (1 + 0.1 * f(H)).astype(np.float32)
q3, k3 = f(R, HQ, D), f(R, HKV, D)
pos = np.array([0, 1, 7, 100, 2047, 5], np.int32)
h_want, y_want = O.residual_rms_norm(x2, r2, w2, 1e-5, impl=O.REF)
h, yy = np.zeros_like(x2), np.zeros_like(x2)
assert L.pin_registry_residual_rms_norm_host(C.c_void_p(P(yy)), C.c_void_p(P(h)), C.c_void_p(P(x2)),
                                             C.c_void_p(P(r2)), C.c_void_p(P(w2)), R, H,
                                             C.c_float(1e-5)) == 0
assert np.array_equal(h, h_want) and np.array_equal(yy, y_want)
act = np.zeros_like(g2)
assert L.pin_registry_swiglu_host(C.c_void_p(P(act)), C.c_void_p(P(g2)), C.c_void_p(P(u2)), R, I) == 0
assert np.array_equal(act, O.swiglu(g2, u2, impl=O.REF))
lg = f(R, 1001)
lg[2, :] = 1.0  # ties: the first maximum
lg[3, 0] = np.float32("nan")  # NaN at 0 keeps 0
tok = np.full(R, -1, np.int32)
assert L.pin_registry_argmax_host(C.c_void_p(P(tok)), C.c_void_p(P(lg)), R, 1001) == 0
assert np.array_equal(tok, O.argmax(lg, impl=O.REF))
qw, kw = O.rope(q3, k3, pos, 1e4, impl=O.REF)
q, k = q3.copy(), k3.copy()
assert L.pin_registry_rope_rows_host(C.c_void_p(P(q)), C.c_void_p(P(k)), C.c_void_p(P(pos)), R,
                                     HQ, HKV, D, C.c_float(1e4)) == 0
assert np.array_equal(q, qw) and np.array_equal(k, kw)
q, k = q3.copy(), k3.copy()
h, yy, act = np.zeros_like(x2), np.zeros_like(x2), np.zeros_like(g2)
assert L.pin_registry_layer_chain_host(*[C.c_void_p(P(a)) for a in (yy, h, act, x2, r2, w2, q, k,
                                                                      g2, u2, pos)],
                                       R, H, HQ, HKV, D, I, C.c_float(1e-5), C.c_float(1e4)) == 0
assert np.array_equal(h, h_want) and np.array_equal(yy, y_want)
assert np.array_equal(q, qw) and np.array_equal(k, kw)
assert np.array_equal(act, O.swiglu(g2, u2, impl=O.REF))
print("ok")
'''
    out = subprocess.run([sys.executable, "-c", code, PIN_REGISTRY_SO, ROOT,
                          os.path.join(ROOT, "tensorbit-run_b200")],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-3000:]


def test_tbm_load_rejects_bad_files_before_device_work(tmp_path):
    """tb_b200_tbm_load checks the container before it touches a device, as
    tb_model_load_tbm does (src/model.c:482-545): a missing file
    (TB_ERR_FILE_OPEN 1), a file too short or whose index length does not fit
    (TB_ERR_TRUNCATED 11), an index that is not JSON (TB_ERR_JSON_PARSE 13),
    and a tensor header or tensor bytes past the end of the file (11)."""
    import json
    import struct
    L = T.lib()
    h = C.c_void_p()

    def load(p):
        return L.tb_b200_tbm_load(str(p).encode(), None, C.byref(h))

    assert load(tmp_path / "missing.tbm") == 1
    (tmp_path / "short.tbm").write_bytes(b"x" * 10)
    assert load(tmp_path / "short.tbm") == 11
    (tmp_path / "len.tbm").write_bytes(b"\0" * 60 + struct.pack("<I", 1000))
    assert load(tmp_path / "len.tbm") == 11
    js = b"{not json"
    (tmp_path / "json.tbm").write_bytes(b"\0" * 64 + js + struct.pack("<I", len(js)))
    assert load(tmp_path / "json.tbm") == 13

    def container(tensors, body=b""):
        js = json.dumps({"architecture": "llama", "config": {"hidden_size": 8},
                         "tensors": tensors}).encode()
        return body + js + struct.pack("<I", len(js))

    t = {"name": "a", "offset": 10 ** 6, "shape": [2, 2], "dtype": "fp32", "num_weights": 4,
         "num_mask_bytes": 0}
    (tmp_path / "off.tbm").write_bytes(container([t]))
    assert load(tmp_path / "off.tbm") == 11
    hdr = struct.pack("<IIIIQQQQB", 0x31304254, 1, 0, 0, 4, 0, 4096, 4096 + 16, 0)
    hdr += b"\0" * (4096 - len(hdr))
    t = dict(t, offset=0, num_weights=10 ** 7)  # 40 MB of weights in a 4 KB file
    (tmp_path / "big.tbm").write_bytes(container([t], hdr + b"\0" * 16))
    assert load(tmp_path / "big.tbm") == 11
    assert not h.value
    assert L.tb_b200_tbm_load(None, None, C.byref(h)) == 8
