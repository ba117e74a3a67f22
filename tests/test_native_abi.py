"""The C-ABI library loads, exports every function the header declares, and
the ctypes mirrors have the header's layout (no GPU needed)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from devproc_b200 import _native as N

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "devproc_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^int\s+(dp_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_what_the_binding_binds():
    assert declared_functions() == sorted(N.EXPORTS)


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.dp_version() // 10000 == 1


def test_last_error_roundtrip_without_gpu():
    # A null-params call fails on the host before touching CUDA.
    st = N.lib().dp_preproc(None, None, None, None)
    assert st == N.DP_ERR_ARG
    assert "null params" in N.last_error()


def test_plan_validation_rejects_garbage_without_gpu():
    h = ctypes.c_void_p()
    st = N.lib().dp_program_create(b"\0" * 64, 64, 0, ctypes.byref(h))
    assert st == N.DP_ERR_PLAN and "magic" in N.last_error()


STRUCTS = {"dp_preproc_params": N.PreprocParams, "dp_rowreduce_params": N.RowReduceParams,
           "dp_gemm_params": N.GemmParams, "dp_region_desc": N.RegionDesc, "dp_embedding_params": N.EmbeddingParams,
           "dp_attention_params": N.AttentionParams, "dp_rope_params": N.RopeParams,
           "dp_splitk_params": N.SplitKParams, "dp_argmax_keys_params": N.ArgmaxKeysParams,
           "dp_streamk_params": N.StreamKParams,
           "dp_plan_header": N.PlanHeader, "dp_plan_slot": N.PlanSlot, "dp_plan_record": N.PlanRecord}


def test_ctypes_layouts_match_the_header(tmp_path):
    src = tmp_path / "sizes.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "devproc_b200.h"', "int main(void){"]
    for cname in STRUCTS:
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
    lines.append('printf("rec_params %zu\\n", offsetof(dp_plan_record, params));')
    lines.append('printf("region_consts %zu\\n", offsetof(dp_region_desc, consts));')
    lines.append('printf("gemm_a_dtype %zu\\n", offsetof(dp_gemm_params, a_dtype));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "sizes"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines())
    for cname, cls in STRUCTS.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
    assert int(got["rec_params"]) == N.PlanRecord.params.offset
    assert int(got["region_consts"]) == N.RegionDesc.consts.offset
    assert int(got["gemm_a_dtype"]) == N.GemmParams.a_dtype.offset
    assert ctypes.sizeof(N.RegionDesc) <= N.DP_RECORD_PARAM_BYTES
