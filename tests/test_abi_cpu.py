"""C-ABI library: loads, exports every symbol the header declares, rejects bad args on the host.

No GPU compute is launched here: every call below fails its host-side argument check
(or is a pure size query) before anything touches a device.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from tasft_b200 import _lib as L

HEADER = Path(__file__).resolve().parent.parent / "include" / "tasft_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TASFT_API\s+[\w\s\*]+?\b(tasft_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    for name in ["tasft_gate_mask_build", "tasft_bsa_prefill_fwd", "tasft_bsa_decode_fwd",
                 "tasft_bsa_decode_combine", "tasft_gate_target_fwd", "tasft_gate_loss_fwd_bwd",
                 "tasft_gate_bwd", "tasft_status_string", "tasft_abi_version"]:
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) == set(L.SIGNATURES), "ctypes signatures out of sync with the header"


def test_abi_version_and_status_strings():
    lib = L.lib()
    assert lib.tasft_abi_version() == 3
    assert lib.tasft_status_string(0) == b"ok"
    assert b"argument" in lib.tasft_status_string(-1)
    assert lib.tasft_launch_count() >= 0


def test_null_args_rejected_on_host():
    lib = L.lib()
    for fn in ["tasft_gate_mask_build", "tasft_mask_from_scores", "tasft_mask_to_kept", "tasft_bsa_prefill_fwd",
               "tasft_bsa_decode_fwd", "tasft_bsa_decode_combine", "tasft_gate_target_fwd",
               "tasft_gate_loss_fwd_bwd", "tasft_gate_bwd"]:
        assert getattr(lib, fn)(None, None) == -1, fn


def test_prefill_bad_shapes_rejected():
    lib = L.lib()
    a = L.PrefillArgs(q=16, k=16, v=16, out=16, B=1, Hq=3, Hk=2, S=64, D=64, block=64, dtype=L.BF16,
                      kept_idx=16, kept_cnt=16, Hm=3)
    for i in range(4):
        a.q_stride[i] = a.k_stride[i] = a.v_stride[i] = a.o_stride[i] = 1
    assert lib.tasft_bsa_prefill_fwd(C.byref(a), None) == -1  # Hq % Hk != 0
    a.Hk = 1
    a.block = 48
    assert lib.tasft_bsa_prefill_fwd(C.byref(a), None) == -2  # block size


def test_workspace_sizes():
    lib = L.lib()
    rows = 4 * 32 * 64 + 4 * 8 * 64
    assert lib.tasft_gate_workspace_size(4, 32, 8, 4096, 4096, 64, 32, 128) == rows * 32 * 4 + rows * 128 * 4
    assert lib.tasft_gate_workspace_size(0, 1, 1, 1, 1, 1, 1, 64) == -1
    assert lib.tasft_decode_workspace_size(64, 32, 8, 128, 4) >= 64 * 32 * 4 * 130 * 4
    assert lib.tasft_gate_target_workspace_size(4, 32, 4096, 64) == 4 * 32 * 64 * 64 * 4
    assert lib.tasft_gate_loss_workspace_size(4, 32) > 0
    assert lib.tasft_gate_bwd_workspace_size(1, 2, 1, 3, 3, 8) > 0


def test_decode_workspace_too_small():
    lib = L.lib()
    a = L.DecodeArgs(q=16, k_cache=16, v_cache=16, out=16, B=2, Hq=4, Hk=2, L=128, D=64, block=64,
                     dtype=L.BF16, kv_len=16, kept_idx=16, kept_cnt=16, nb_max=2, num_splits=2,
                     workspace=16, workspace_bytes=8)
    a.q_stride[0], a.q_stride[1], a.q_stride[2] = 256, 64, 1
    for st in (a.k_stride, a.v_stride):
        st[0], st[1], st[2], st[3] = 2 * 128 * 64, 128 * 64, 64, 1
    a.o_stride[0], a.o_stride[1], a.o_stride[2] = 256, 64, 1
    assert lib.tasft_bsa_decode_fwd(C.byref(a), None) == -4


def test_check_raises_kernel_error():
    from tasft_b200.exceptions import KernelError, ValidationError
    with pytest.raises(ValidationError):
        L.check(-1, "x")
    with pytest.raises(KernelError):
        L.check(-2, "x")


# ctypes mirrors of the header's structs: every field's offset and every struct's size,
# as gcc lays them out from include/tasft_b200.h (a drift would corrupt calls silently)
_STRUCTS = {
    "tasft_gate_args": "GateArgs", "tasft_threshold_args": "ThresholdArgs", "tasft_mask_args": "MaskArgs",
    "tasft_prefill_args": "PrefillArgs", "tasft_prefill_varlen_args": "PrefillVarlenArgs",
    "tasft_decode_args": "DecodeArgs", "tasft_paged_decode_args": "PagedDecodeArgs",
    "tasft_combine_args": "CombineArgs", "tasft_target_args": "TargetArgs", "tasft_loss_args": "LossArgs",
    "tasft_gate_bwd_args": "GateBwdArgs",
}


def test_struct_layouts_match_header(tmp_path):
    import ctypes as C  # noqa: PLC0415
    import shutil  # noqa: PLC0415
    import subprocess  # noqa: PLC0415

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    lines = ["#include <stddef.h>", "#include <stdio.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, pyname in _STRUCTS.items():
        cls = getattr(L, pyname)
        lines.append(f'  printf("{pyname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{pyname}.{field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c11", "-o", str(exe), str(src)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                                check=True).stdout.splitlines())
    for pyname in _STRUCTS.values():
        cls = getattr(L, pyname)
        assert int(got[f"{pyname} size"]) == C.sizeof(cls), pyname
        for field, _ in cls._fields_:
            assert int(got[f"{pyname}.{field}"]) == getattr(cls, field).offset, f"{pyname}.{field}"
