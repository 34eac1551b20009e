"""The Rust binding (rust/burn_jepa_b200) against the C ABI, on the CPU.

cargo/rustc are not in this image, so the crate is not compiled here; this test parses its
`extern "C"` block and checks every declaration against include/bjf.h: the same set of entry
points, and per function the same arity and, argument by argument and for the return value,
the same kind and width (pointer / i32 / i64 / u64 / usize / f32), plus the #[repr(C)] struct
fields and the ABI version constant."""
import os
import re

from burn_jepa_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FFI = os.path.join(ROOT, "rust", "burn_jepa_b200", "src", "ffi.rs")

C_SCALARS = {"int32_t": "i32", "uint32_t": "u32", "bjf_status": "i32", "bjf_dtype": "i32", "int64_t": "i64", "uint64_t": "u64",
             "size_t": "usize", "float": "f32", "void": "void"}
RUST_SCALARS = {"i32": "i32", "u32": "u32", "bjf_status": "i32", "bjf_dtype": "i32", "i64": "i64", "u64": "u64", "usize": "usize",
                "f32": "f32"}


def _c_kind(decl: str) -> str:
    decl = decl.strip()
    if "*" in decl or "[" in decl or decl.startswith("bjf_stream_t"):
        return "ptr"
    base = decl.replace("const ", "").split()[0]
    return C_SCALARS[base]


def _rust_kind(ty: str) -> str:
    ty = ty.strip()
    if ty.startswith("*") or ty == "bjf_stream_t":
        return "ptr"
    return RUST_SCALARS[ty]


def c_functions():
    text = re.sub(r"/\*.*?\*/", "", open(_abi.HEADER_PATH).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"BJF_API\s+([\w\s\*]+?)\b(bjf_\w+)\s*\((.*?)\);", text, re.S):
        args = [a for a in " ".join(m.group(3).split()).split(",") if a.strip() and a.strip() != "void"]
        out[m.group(2)] = (_c_kind(m.group(1)), [_c_kind(a) for a in args])
    return out


def rust_functions():
    text = open(FFI).read()
    block = re.search(r'extern "C"\s*\{(.*?)\n\}', text, re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (bjf_\w+)\s*\((.*?)\)\s*(?:->\s*([\w\*\s]+?))?\s*;", block, re.S):
        args = [a for a in " ".join(m.group(2).split()).split(",") if a.strip()]
        kinds = [_rust_kind(a.split(":", 1)[1]) for a in args]
        out[m.group(1)] = (_rust_kind(m.group(3)) if m.group(3) else "void", kinds)
    return out


def test_ffi_declares_every_entry_point_of_the_header():
    c, r = c_functions(), rust_functions()
    assert sorted(c) == sorted(r), (sorted(set(c) ^ set(r)))
    assert sorted(c) == _abi.header_symbols()


def test_ffi_signatures_match_the_header():
    c, r = c_functions(), rust_functions()
    for name in c:
        assert r[name][0] == c[name][0], f"{name}: return {r[name][0]} vs {c[name][0]}"
        assert len(r[name][1]) == len(c[name][1]), f"{name}: arity {len(r[name][1])} vs {len(c[name][1])}"
        for i, (a, b) in enumerate(zip(r[name][1], c[name][1])):
            assert a == b, f"{name}: argument {i} is {a} in ffi.rs, {b} in bjf.h"


def _c_struct_fields(name):
    text = re.sub(r"/\*.*?\*/", "", open(_abi.HEADER_PATH).read(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, text, re.S).group(1)
    fields = []
    for line in body.split(";"):
        line = line.strip()
        if not line:
            continue
        if "*" in line:  # a device pointer
            fields.append((line.split("*")[-1].strip(), "ptr", 1))
            continue
        m = re.match(r"([\w\s]+?)\s+(\w+)(\[(\d+)\])?$", line)
        ty, field, _, n = m.groups()
        ty = ty.strip()
        kind = "struct" if ty.startswith("bjf_") and ty not in ("bjf_dtype",) else C_SCALARS[ty]
        fields.append((field, kind, int(n) if n else 1))
    return fields


def _rust_struct_fields(name):
    body = re.search(r"pub struct %s \{(.*?)\}" % name, open(FFI).read(), re.S).group(1)
    fields = []
    for m in re.finditer(r"pub (\w+):\s*([^,]+),", body):
        field, ty = m.groups()
        ty = ty.strip()
        arr = re.match(r"\[(\w+);\s*(\d+)\]", ty)
        if ty.startswith("*"):
            fields.append((field, "ptr", 1))
        elif arr:
            fields.append((field, RUST_SCALARS[arr.group(1)], int(arr.group(2))))
        elif ty.startswith("bjf_") and ty != "bjf_dtype":
            fields.append((field, "struct", 1))
        else:
            fields.append((field, RUST_SCALARS[ty], 1))
    return fields


def test_ffi_structs_match_the_header():
    for name in ("bjf_patchify_config", "bjf_patch_diff_config", "bjf_rgba_frame_stats", "bjf_viewer_mask_policy",
                 "bjf_patch_diff_refresh_config", "bjf_patch_diff_refresh_state", "bjf_front_end_desc"):
        assert _rust_struct_fields(name) == _c_struct_fields(name), name


def test_ffi_abi_version_matches_the_header():
    m = re.search(r"pub const BJF_ABI_VERSION: i32 = (\d+);", open(FFI).read())
    assert int(m.group(1)) == _abi.header_abi_version()
