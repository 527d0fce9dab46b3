"""CPU checks of the C-ABI library: it loads, exports every entry point that
include/qic.h and include/qic_kernels_compat.h declare, and rejects invalid
arguments before touching a device."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared_c_functions():
    text = (ROOT / "include" / "qic.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(qic_\w+)\s*\(", text, re.M)))


def _exported():
    from qwenincuda_b200 import lib_path

    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path())], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}


def test_library_loads():
    import qwenincuda_b200 as q

    L = q.lib()
    assert L.qic_version() >= 100


def test_every_declared_symbol_is_exported():
    names = _declared_c_functions()
    assert len(names) >= 12, names
    exported = _exported()
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_compat_symbols_exported():
    """The C++ surface of the reference's include/kernels.cuh, mangled with `half`."""
    text = (ROOT / "include" / "qic_kernels_compat.h").read_text()
    names = re.findall(r"^void (launch_\w+)\(", text, re.M)
    assert len(names) == 10
    exported = _exported()
    for n in names:
        assert any(re.fullmatch(rf"_Z\d+{n}P.*6__half.*", s) for s in exported), n
    assert "qic_compat_last_status" in exported


def test_status_strings():
    import qwenincuda_b200 as q

    L = q.lib()
    assert L.qic_status_string(0) == b"success"
    for s in range(1, 9):
        assert L.qic_status_string(s) not in (b"success", b"unknown status")


def test_workspace_bytes():
    import qwenincuda_b200 as q

    L = q.lib()
    assert L.qic_decode_workspace_bytes(0, 8, 128, 10) == 0
    b1 = L.qic_decode_workspace_bytes(32, 8, 128, 8192)
    b2 = L.qic_decode_workspace_bytes(32, 8, 128, 16)
    assert b1 > b2 > 256


def test_argument_validation_without_device():
    import qwenincuda_b200 as q

    L = q.lib()
    a = q.DecodeArgs()
    assert L.qic_decode_attention(None, None) == 1
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # zero heads
    a.dtype, a.num_heads, a.num_kv_heads, a.head_dim, a.seq_len = 1, 32, 8, 96, 10
    a.q = a.k_cache = a.v_cache = a.out = 0x10000
    a.cache_tokens = 100
    assert L.qic_decode_attention(ctypes.byref(a), None) == 2          # head_dim 96
    a.head_dim = 128
    a.num_kv_heads = 3
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # 32 % 3
    a.num_kv_heads = 2
    assert L.qic_decode_attention(ctypes.byref(a), None) == 2          # group 16 > 8
    a.num_kv_heads = 8
    a.k_cache = 0x10008
    assert L.qic_decode_attention(ctypes.byref(a), None) == 3          # misaligned cache
    a.k_cache = 0x10000
    a.page_table = 0x20000
    a.page_size = 12
    assert L.qic_decode_attention(ctypes.byref(a), None) == 2          # page size not a multiple of 8
    a.page_table = None
    a.seq_len = 200
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # S > cache_tokens (contiguous)
    g = q.GdnArgs()
    assert L.qic_gated_delta_decode(ctypes.byref(g), None) == 1
    g.dtype, g.num_k_heads, g.num_v_heads, g.k_head_dim, g.v_head_dim, g.conv_kernel = 1, 16, 32, 64, 128, 4
    assert L.qic_gated_delta_decode(ctypes.byref(g), None) == 2
    assert L.qic_kv_append(1, None, None, None, 1e-6, 1e6, 0, None, None, None, 16, 10, 8, 128, None) == 1
    a.seq_len = 10
    a.flags = q.abi.QIC_Q_GATE_INTERLEAVED
    a.gate = 0x30000
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # gate given twice (interleaved q)
    a.flags = q.abi.QIC_DEVICE_SEQ_LEN
    a.gate = None
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # device length without its pointer
    a.seq_len_dev = 0x40002
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # misaligned length pointer
    a.seq_len_dev = 0x40000
    assert L.qic_decode_attention(ctypes.byref(a), None) == 1          # device length without a workspace


def test_header_constants_match_bindings():
    """Every QIC_* enum value of include/qic.h has the same value in the ctypes bindings."""
    from qwenincuda_b200 import abi

    text = (ROOT / "include" / "qic.h").read_text()
    consts = dict(re.findall(r"\b(QIC_[A-Z0-9_]+)\s*=\s*(\d+)", text))
    consts.update(re.findall(r"#define\s+(QIC_[A-Z0-9_]+)\s+(\d+)", text))
    assert len(consts) >= 20
    for name, value in consts.items():
        if name.startswith("QIC_ERROR_") or name == "QIC_SUCCESS":
            assert abi.STATUS_NAMES[int(value)] == name
        else:
            assert getattr(abi, name) == int(value), name


def test_libraries_bind_their_own_symbols():
    """libqic.so exports the kernels.cuh C++ names and so does the reference's fp16
    build; both are linked -Bsymbolic so neither library's internal calls can be
    bound to the other's same-named functions when both are loaded in one process."""
    from qwenincuda_b200 import lib_path

    libs = [lib_path()] + sorted((ROOT / "oracle" / "_ref").glob("libqicref_*.so"))
    for p in libs:
        out = subprocess.run(["readelf", "-d", str(p)], capture_output=True, text=True, check=True).stdout
        assert "SYMBOLIC" in out, p


def test_struct_layouts_match_the_header(tmp_path):
    """Every ctypes mirror has the C struct's size and every field its C offset: a C
    program compiled against include/qic.h prints them (gcc, no GPU)."""
    from qwenincuda_b200 import abi

    mirrors = {"qic_decode_args": abi.DecodeArgs, "qic_cp_args": abi.CpArgs,
               "qic_batch_decode_args": abi.BatchDecodeArgs, "qic_gdn_args": abi.GdnArgs}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "qic.h"', "int main(void) {"]
    for cname, cls in mirrors.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        cname, field, value = line.split()
        got[(cname, field)] = int(value)
    for cname, cls in mirrors.items():
        assert ctypes.sizeof(cls) == got[(cname, "sizeof")], cname
        for field, _ in cls._fields_:
            assert getattr(cls, field).offset == got[(cname, field)], f"{cname}.{field}"
