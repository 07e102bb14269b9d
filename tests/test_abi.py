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
