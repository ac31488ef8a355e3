"""The C ABI: symbols, error statuses, NVRTC compile -- no GPU needed."""
import ctypes
import os
import re

import numpy as np
import pytest

from nablatensor_b200 import _lib, quant
from nablatensor_b200.tape import AadRecorder

from tapes import every_op_tape, multi_output, named_streams, nonuniform_asian, pow2_divisions, term_vol_asian

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "nabla_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nt_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(ntlib):
    declared = _declared()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(ntlib, name), name
    assert sorted(_lib.SIGNATURES) == declared


def test_version_and_device_probe_never_fault(ntlib):
    assert ntlib.nt_version() == 1
    n = _lib.device_count()  # 0 on a CPU-only machine, no exception
    assert n >= 0


def _compile_status(tape, **opts):
    s, keep = _lib.tape_struct(tape)
    o = _lib.options_struct(**opts)
    h = ctypes.c_void_p()
    rc = _lib.lib().nt_compile(ctypes.byref(s), ctypes.byref(o), ctypes.byref(h))
    msg = _lib.lib().nt_last_error().decode()
    if rc == 0:
        _lib.lib().nt_destroy(h)
    return rc, msg


def _tape_arrays(tape):
    return {k: np.array(getattr(tape, k)) for k in
            ("op", "arg_a", "arg_b", "constant", "input_node", "output_node", "normal_count", "uniform_count")}


class _Raw:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def _malformed(mutate):
    t = quant.asian_tape(8)
    d = _tape_arrays(t)
    mutate(d)
    return _Raw(**d)


@pytest.mark.parametrize("mutate,needle", [
    (lambda d: d["op"].__setitem__(20, 99), "unknown op"),
    (lambda d: d["arg_a"].__setitem__(20, 10_000), "out of order"),
    (lambda d: d["arg_b"].__setitem__(22, 22), "out of order"),
    (lambda d: d["arg_a"].__setitem__(0, 7), "input index out of range"),
    (lambda d: d["arg_a"].__setitem__(15, 3), "draw ordinals"),
    (lambda d: d["arg_b"].__setitem__(15, 4), "stream out of range"),
    (lambda d: d["output_node"].__setitem__(0, 10**6), "out of range"),
    (lambda d: d["input_node"].__setitem__(1, 5), "is not INPUT"),
    (lambda d: d["normal_count"].__setitem__(0, 3), "normal_count"),
])
def test_malformed_tapes_are_rejected_before_emission(ntlib, mutate, needle):
    """ingest() checks every index (the reference trusted its recorder)."""
    raw = _malformed(mutate)
    s, keep = _lib.tape_struct(raw)
    o = _lib.options_struct()
    n = ctypes.c_size_t(0)
    rc = _lib.lib().nt_emit_source(ctypes.byref(s), ctypes.byref(o), 0, None, 0, ctypes.byref(n))
    assert rc == _lib.NT_E_TAPE
    assert needle in _lib.lib().nt_last_error().decode()


def test_invalid_arguments(ntlib):
    L = _lib.lib()
    assert L.nt_compile(None, None, None) == _lib.NT_E_INVALID_ARG
    assert L.nt_replay(None, 1, 0, 0, None, None) == _lib.NT_E_STATE
    assert "closed" in L.nt_last_error().decode()
    L.nt_destroy(None)  # no-op
    f, c = ctypes.c_uint64(), ctypes.c_uint64()
    assert L.nt_shard_range(10, 0, 0, 0, ctypes.byref(f), ctypes.byref(c)) == _lib.NT_E_INVALID_ARG
    with pytest.raises(_lib.NablaError) as e:
        _lib.emit_source(quant.asian_tape(4), target=4)
    assert e.value.code == _lib.NT_E_INVALID_ARG
    for regs in (8, 256, -1):
        with pytest.raises(_lib.NablaError) as e:
            _lib.emit_source(quant.asian_tape(4), max_regs=regs)
        assert e.value.code == _lib.NT_E_INVALID_ARG and "max_regs" in str(e.value)
    for key, bad in (("fwd_unroll", 17), ("fwd_unroll", -1), ("rev_unroll", 9), ("rev_unroll", -1)):
        with pytest.raises(_lib.NablaError) as e:
            _lib.emit_source(quant.asian_tape(4), **{key: bad})
        assert e.value.code == _lib.NT_E_INVALID_ARG and key in str(e.value)


def test_bad_block_size_is_an_argument_error(ntlib):
    rc, msg = _compile_status(quant.asian_tape(4), block=100)
    # on a CPU box the device probe may fail first; either way no fault
    assert rc in (_lib.NT_E_INVALID_ARG, _lib.NT_E_CUDA)


@pytest.mark.parametrize("f32", [False, True])
@pytest.mark.parametrize("make", [lambda: quant.asian_tape(252), lambda: quant.barrier_tape(252), every_op_tape,
                                  lambda: named_streams(16), lambda: multi_output(40)])
def test_emitted_kernels_compile_for_sm100a(ntlib, make, f32):
    src = _lib.emit_source(make(), target=0, precision=0 if f32 else 1)
    assert "nt_replay_kernel" in src and "__launch_bounds__" in src
    assert _lib.nvrtc_check(src) > 1000


@pytest.mark.parametrize("make,f32", [(lambda: quant.asian_tape(252), False), (lambda: quant.barrier_tape(252), True),
                                      (lambda: quant.basket_tape(), False), (every_op_tape, False)])
def test_multi_market_kernels_compile_for_sm100a(ntlib, make, f32):
    src = _lib.emit_source(make(), target=2, precision=0 if f32 else 1)
    assert "nt_markets_kernel" in src and "nt_grid_reduce_cols" in src
    assert _lib.nvrtc_check(src) > 1000


def test_nvrtc_errors_are_reported(ntlib):
    with pytest.raises(_lib.NablaError) as e:
        _lib.nvrtc_check("extern \"C\" __global__ void k() { this is not C++; }")
    assert e.value.code == _lib.NT_E_NVRTC
    assert "NVRTC compile failed" in str(e.value)


def test_shard_ranges_tile_the_range(ntlib):
    for total in (1, 7, 2_000_000, 10**9 + 3):
        for n in (1, 2, 3, 8):
            cur = 123
            for r in range(n):
                f, c = _lib.shard_range(total, 123, n, r)
                assert f == cur
                cur += c
            assert cur == 123 + total


def test_inputs_without_a_device_fail_loudly(ntlib):
    """No CPU fallback: compiling on a machine without a B200 is an error."""
    if _lib.device_count() > 0:
        pytest.skip("a GPU is present")
    rc, msg = _compile_status(quant.asian_tape(8))
    assert rc != 0 and msg


def test_recorded_tapes_round_trip_through_the_abi(ntlib):
    t = AadRecorder.record(lambda rec: rec.output(rec.input("x", 1.0).mul(2.0)))
    src = _lib.emit_source(t, target=1)
    assert "nt_host_replay" in src


def _header_fields(struct: str):
    with open(os.path.join(ROOT, "include", "nabla_b200.h")) as f:
        text = f.read()
    body = re.search(r"typedef struct " + struct + r" \{(.*?)\} " + struct + ";", text, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return [re.search(r"(\w+)\s*;", line).group(1) for line in body.split("\n") if ";" in line]


@pytest.mark.parametrize("struct,cls", [("nt_tape", _lib.NtTape), ("nt_options", _lib.NtOptions),
                                        ("nt_exec_info", _lib.NtExecInfo)])
def test_ctypes_layouts_follow_the_header(struct, cls):
    assert [name for name, _ in cls._fields_] == _header_fields(struct)


def test_math_eval_rejects_bad_arguments_before_touching_a_device(ntlib):
    L = _lib.lib()
    out = np.zeros(4)
    x = np.zeros(4)
    p = out.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
    xp = x.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
    assert L.nt_math_eval(0, 8, 4, None, xp, p, p) == _lib.NT_E_INVALID_ARG  # unknown routine
    assert L.nt_math_eval(0, 2, 0, None, xp, p, None) == _lib.NT_E_INVALID_ARG  # n < 1
    assert L.nt_math_eval(0, 2, (1 << 24) + 1, None, xp, p, None) == _lib.NT_E_INVALID_ARG  # n > 2^24
    assert L.nt_math_eval(0, 0, 4, None, xp, p, None) == _lib.NT_E_INVALID_ARG  # words needed
    assert L.nt_math_eval(0, 1, 4, None, xp, p, None) == _lib.NT_E_INVALID_ARG  # out1 needed


@pytest.mark.parametrize("target", [0, 2])
@pytest.mark.parametrize("make,opts", [
    (lambda: quant.cva_tape(), {}),                      # gathered curve (shared memory), per-date table, carried leg
    (term_vol_asian, {}),                                # gathered per-step inputs
    (nonuniform_asian, {}),                              # per-unit constant table
    (pow2_divisions, {}),                                # divisions rewritten as multiplications
    (lambda: quant.basket_tape(), {"seg_units": 2}),     # the two-unit segment the engine may pick
    (lambda: quant.asian_tape(252), {"rev_unroll": 2}),  # unrolled reverse segment loop
])
def test_plan_features_compile_for_sm100a(ntlib, make, opts, target):
    """Every emission feature of the planner, for the single- and the
    multi-market kernel, compiles with NVRTC for sm_100a."""
    src = _lib.emit_source(make(), target=target, **opts)
    assert ("nt_markets_kernel" if target == 2 else "nt_replay_kernel") in src
    assert _lib.nvrtc_check(src) > 1000


def _segments(src):
    m = re.search(r"step loop: (\d+) units of \d+ nodes \(\d+ steps each\), (\d+) segments of (\d+) units", src)
    return int(m.group(1)), int(m.group(2)), int(m.group(3))


def test_automatic_segment_lengths(ntlib):
    """fp64 tapes with a value tape plan segments within about 112 registers,
    the rest within 64: the Asian gets 9 units, the fp32 barrier 3, the heavy
    basket and CVA units 1, the recompute-all Asian 6."""
    asian = quant.asian_tape(252)
    assert _segments(_lib.emit_source(asian)) == (126, 14, 9)
    rc = _lib.NT_FLAG_RECOMPUTE_ALL | _lib.NT_FLAG_SHARED_CKPT
    assert _segments(_lib.emit_source(asian, flags=rc)) == (126, 21, 6)
    assert _segments(_lib.emit_source(quant.barrier_tape(252), precision=_lib.NT_FLOAT32)) == (126, 42, 3)
    assert _segments(_lib.emit_source(quant.basket_tape()))[2] == 1
    assert _segments(_lib.emit_source(quant.cva_tape()))[2] == 1


def test_l2_discard_of_consumed_tape_rows_is_placed_safely(ntlib):
    """discard.global.L2 of a consumed tape segment is emitted only where a
    light unit's tape can stay in L2, under the kernel's run-time check that
    the grid's tape fits, and only in the last output's reverse sweep: an
    earlier output's sweep reads the same rows again."""
    def sweeps(src):
        return [m.start() for m in re.finditer(r"reverse sweep, output (\d+)", src)]

    src = _lib.emit_source(quant.asian_tape(252))
    assert "const bool nt_tape_in_l2 =" in src
    # one per reverse copy (series and guarded), each inside `if (nt_tape_in_l2)`
    assert src.count("nt_discard_rows_l2<") == 2
    assert src.count("if (nt_tape_in_l2) {") == 2
    two = _lib.emit_source(multi_output(40))
    starts = sweeps(two)
    assert len(starts) == 2
    hits = [m.start() for m in re.finditer(r"nt_discard_rows_l2<", two)]
    assert hits and all(h > starts[1] for h in hits)
    # heavy units, recompute-all, the host build and the multi-market kernel: none
    rc = _lib.NT_FLAG_RECOMPUTE_ALL | _lib.NT_FLAG_SHARED_CKPT
    # and the fp32 barrier, whose tape (3 KB per thread) cannot fit even at one block per SM
    barrier = _lib.emit_source(quant.barrier_tape(252), precision=_lib.NT_FLOAT32)
    for src in (barrier, _lib.emit_source(quant.cva_tape()), _lib.emit_source(quant.basket_tape()),
                _lib.emit_source(quant.asian_tape(252), flags=rc), _lib.emit_source(quant.asian_tape(252), target=1),
                _lib.emit_source(quant.asian_tape(252), target=2)):
        assert "nt_discard_rows_l2<" not in src


def test_a_missing_library_fails_loudly_and_the_engine_reports_unavailable(monkeypatch):
    """No fallback: without libnabla_b200.so every entry raises, and the SPI's
    isAvailable() answers False without throwing (AadEngine.java:39-40)."""
    from nablatensor_b200.engine import CudaAadEngine
    monkeypatch.setattr(_lib, "LIB_PATH", os.path.join(ROOT, "no_such_dir", "libnabla_b200.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="is missing"):
        _lib.lib()
    assert CudaAadEngine(0).isAvailable() is False


def test_the_engine_compiles_with_the_toolkit_nvrtc_whatever_the_host_loaded_first():
    """The engine loads the CUDA toolkit's NVRTC privately, by path.  A host
    that has already loaded another libnvrtc.so.12 -- torch imports its own
    bundled copy -- must not change the compiler, since two NVRTC versions may
    fuse a multiply-add differently and so change an fp32 kernel's sums."""
    import subprocess
    import sys
    probe = ("import ctypes, sys\n"
             "if sys.argv[1] == 'torch-first':\n"
             "    import torch  # noqa: F401  (loads its own libnvrtc.so.12)\n"
             "from nablatensor_b200 import _lib\n"
             "print('%d.%d %s' % _lib.nvrtc_version())\n")
    env = dict(os.environ, PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    env.pop("NT_NVRTC_LIBRARY", None)
    seen = [subprocess.run([sys.executable, "-c", probe, mode], capture_output=True, text=True, env=env,
                           timeout=300, check=True).stdout.strip() for mode in ("alone", "torch-first")]
    assert seen[0] == seen[1], seen
    version, path = seen[0].split(" ", 1)
    assert os.path.isabs(path) and "libnvrtc.so" in path, path
    assert "site-packages" not in path, path


def test_a_missing_nvrtc_is_an_error_status_not_a_crash():
    """NT_NVRTC_LIBRARY naming a file that does not exist: compiling fails
    with NT_E_NVRTC and a message naming the file."""
    import subprocess
    import sys
    probe = ("from nablatensor_b200 import _lib, quant\n"
             "try:\n"
             "    _lib.nvrtc_check(_lib.emit_source(quant.asian_tape(4), 0))\n"
             "    print('compiled')\n"
             "except _lib.NablaError as e:\n"
             "    print(e.code == _lib.NT_E_NVRTC, str(e))\n")
    env = dict(os.environ, PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
               NT_NVRTC_LIBRARY="/nonexistent/libnvrtc.so.12")
    out = subprocess.run([sys.executable, "-c", probe], capture_output=True, text=True, env=env, timeout=300,
                         check=True).stdout
    assert out.startswith("True") and "/nonexistent/libnvrtc.so.12" in out, out
