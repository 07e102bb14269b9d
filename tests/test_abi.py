"""The C ABI: the library loads without a GPU, exports every function the header declares,
and the ctypes mirrors of the header's structs have the C compiler's sizes and offsets."""
import ctypes
import re
import shutil
import subprocess

import pytest

from conftest import REPO
from namitorch_b200 import _build
from namitorch_b200 import _native as N

HEADER = REPO / "include" / "namitorch_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(nt_\w+)\s*\(", text, flags=re.M)))


def test_library_is_built_and_current():
    _build.build()
    assert _build.LIB_PATH.exists()
    assert not _build.is_stale()


def test_every_declared_symbol_is_exported_and_bound():
    lib = N.load()
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
        assert name in N.SIGNATURES, f"{name} has no ctypes signature"
    assert set(N.SIGNATURES) == set(names)
    assert lib.nt_abi_version() == N.ABI_VERSION


def test_errors_are_reported_without_a_gpu():
    lib = N.load()
    assert lib.nt_adamw_mt(None, None) == N.NT_EINVAL
    assert b"args is NULL" in lib.nt_last_error()
    with pytest.raises(ValueError, match="ten finite float32 coefficients"):
        coef = (ctypes.c_float * 10)(*([float("nan")] + [1.0] * 9))
        N.check(lib.nt_adamw_f32(None, None, None, None, coef, 0, 1, 8, None))
    args = N.ZeroReduceArgs(num_ranks=9)
    assert lib.nt_zero_reduce_scatter_stats(ctypes.byref(args), None) == N.NT_EINVAL
    assert b"num_ranks" in lib.nt_last_error()
    assert lib.nt_adamw_mt_push(None, None, 0, None) == N.NT_EINVAL
    assert lib.nt_ipc_close(ctypes.c_void_p(16)) == N.NT_EINVAL
    with pytest.raises(ValueError, match="label_smoothing"):
        args = N.XentArgs(rows=1, classes=4, dtype=N.NT_BF16, label_smoothing=1.5, reduction=1)
        N.check(lib.nt_softmax_xent(ctypes.byref(args), None))


def test_kernel_seams_validate_before_touching_the_gpu():
    """The softmax, normalization and elementwise entry points reject malformed calls (and
    accept empty ones) without a CUDA call, so these run on a machine without a GPU."""
    lib = N.load()
    assert lib.nt_fused_elementwise(None, None) == N.NT_EINVAL
    bad_op = N.FusedArgs(op=99, dtype=N.NT_F32, count=4)
    assert lib.nt_fused_elementwise(ctypes.byref(bad_op), None) == N.NT_EINVAL
    assert b"unknown operation" in lib.nt_last_error()
    ragged = N.FusedArgs(op=N.FUSED_OPS["bias_relu"], dtype=N.NT_F32, count=10, width=4)
    assert lib.nt_fused_elementwise(ctypes.byref(ragged), None) == N.NT_EINVAL
    assert b"width" in lib.nt_last_error()
    unbounded = N.FusedArgs(op=N.FUSED_OPS["clamp"], dtype=N.NT_F32, count=4)
    assert lib.nt_fused_elementwise(ctypes.byref(unbounded), None) == N.NT_EINVAL
    assert b"minimum or a maximum" in lib.nt_last_error()
    double = N.FusedArgs(op=N.FUSED_OPS["silu"], dtype=7, count=4)
    assert lib.nt_fused_elementwise(ctypes.byref(double), None) == N.NT_EUNSUPPORTED
    missing = N.FusedArgs(op=N.FUSED_OPS["swiglu"], dtype=N.NT_BF16, count=8, a=16, output=16)
    assert lib.nt_fused_elementwise(ctypes.byref(missing), None) == N.NT_EINVAL
    assert b"operand b is NULL" in lib.nt_last_error()
    empty = N.FusedArgs(op=N.FUSED_OPS["gelu_tanh"], dtype=N.NT_F16, count=0)
    assert lib.nt_fused_elementwise(ctypes.byref(empty), None) == N.NT_OK
    assert lib.nt_row_softmax(None, None) == N.NT_EINVAL
    assert lib.nt_norm_forward(None, None) == N.NT_EINVAL
    wide = N.NormArgs(op=N.NORM_OPS["layer_norm"], dtype=N.NT_F32, rows=2, width=N.NT_NORM_MAX_WIDTH + 1, eps=1e-5)
    assert lib.nt_norm_forward(ctypes.byref(wide), None) == N.NT_EINVAL
    rms_bias = N.NormArgs(op=N.NORM_OPS["rms_norm"], dtype=N.NT_F32, rows=2, width=8, bias=16, eps=1e-5)
    assert lib.nt_norm_forward(ctypes.byref(rms_bias), None) == N.NT_EINVAL
    assert b"RMS norm takes no bias" in lib.nt_last_error()
    no_eps = N.NormArgs(op=N.NORM_OPS["layer_norm"], dtype=N.NT_F32, rows=2, width=8, input=16, output=16, eps=0.0)
    assert lib.nt_norm_forward(ctypes.byref(no_eps), None) == N.NT_EINVAL
    no_ws = N.NormArgs(op=N.NORM_OPS["layer_norm"], dtype=N.NT_F32, rows=2, width=8, input=16, gradient=16,
                       statistics=16, grad_weight=16)
    assert lib.nt_norm_backward(ctypes.byref(no_ws), None) == N.NT_EINVAL
    assert b"workspace" in lib.nt_last_error()
    lib.nt_norm_workspace_size.restype = ctypes.c_size_t
    assert lib.nt_norm_workspace_size(0, 8) == 0
    assert lib.nt_norm_workspace_size(3, 8) == 3 * 8 * 2 * 4


STRUCTS = {
    "nt_segment": (N.Segment, ["grad", "offset", "count", "chunk_begin", "group", "step_slot"]),
    "nt_adamw_group": (N.AdamWGroup, [f for f, _ in N.AdamWGroup._fields_]),
    "nt_stats": (N.Stats, [f for f, _ in N.Stats._fields_]),
    "nt_adamw_mt_args": (N.AdamWMtArgs, [f for f, _ in N.AdamWMtArgs._fields_]),
    "nt_span": (N.Span, [f for f, _ in N.Span._fields_]),
    "nt_grad_stats_args": (N.GradStatsArgs, [("pass" if f == "pass_" else f) for f, _ in N.GradStatsArgs._fields_]),
    "nt_xent_info": (N.XentInfo, None),
    "nt_xent_args": (N.XentArgs, [f for f, _ in N.XentArgs._fields_]),
    "nt_zero_reduce_args": (N.ZeroReduceArgs, [f for f, _ in N.ZeroReduceArgs._fields_]),
    "nt_lr_entry": (N.LrEntry, [f for f, _ in N.LrEntry._fields_]),
    "nt_softmax_args": (N.SoftmaxArgs, [f for f, _ in N.SoftmaxArgs._fields_]),
    "nt_norm_args": (N.NormArgs, [f for f, _ in N.NormArgs._fields_]),
    "nt_fused_args": (N.FusedArgs, [f for f, _ in N.FusedArgs._fields_]),
    "nt_zero_mailbox": (N.ZeroMailbox, [f for f, _ in N.ZeroMailbox._fields_]),
    "nt_zero_sync": (N.ZeroSync, [f for f, _ in N.ZeroSync._fields_]),
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layouts_match_the_c_compiler(tmp_path):
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "namitorch_b200.h"', "int main(void) {"]
    for cname, (_, fields) in STRUCTS.items():
        lines.append(f'  printf("{cname} %zu\\n", sizeof({cname}));')
        for f in fields or []:
            lines.append(f'  printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                                check=True).stdout.splitlines())
    for cname, (cls, fields) in STRUCTS.items():
        assert int(out[cname]) == ctypes.sizeof(cls), cname
        for cf, (pf, _) in zip(fields or [], cls._fields_):
            assert int(out[f"{cname}.{cf}"]) == getattr(cls, pf).offset, f"{cname}.{cf}"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_operation_codes_match_the_header(tmp_path):
    """The Python operation tables carry the header's enum values."""
    text = HEADER.read_text()
    names = {f"NT_FUSED_{k.upper()}": v for k, v in N.FUSED_OPS.items()}
    names.update({f"NT_{k.upper()}": v for k, v in N.SOFTMAX_OPS.items()})
    names.update({"NT_RMS_NORM": N.NORM_OPS["rms_norm"], "NT_LAYER_NORM": N.NORM_OPS["layer_norm"]})
    for name in names:
        assert re.search(rf"\b{name}\b", text), name
    lines = ["#include <stdio.h>", '#include "namitorch_b200.h"', "int main(void) {"]
    lines += [f'  printf("{n} %d\\n", (int){n});' for n in names]
    lines += ["  return 0;", "}"]
    src = tmp_path / "codes.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "codes"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for name, value in names.items():
        assert int(out[name]) == value, name
