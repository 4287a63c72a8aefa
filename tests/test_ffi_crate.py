"""CPU test of the Rust FFI crate (ffi/src/lib.rs): it is not compiled in this image (no cargo),
so its declarations are checked against include/moe_b200.h as text -- every header function is
declared once in the extern block with the same argument count and types and return type, the
#[repr(C)] structs list the C fields in order with the same types, and the constants agree."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

# C type (normalised) -> Rust type
C2RUST = {
    "int": "i32", "int32_t": "i32", "uint32_t": "u32", "uint64_t": "u64", "uint16_t": "u16",
    "float": "f32", "size_t": "usize", "void": "()",
    "void*": "*mut c_void", "const void*": "*const c_void", "void**": "*mut *mut c_void",
    "moe_ctx*": "*mut MoeCtx", "const moe_ctx*": "*const MoeCtx", "moe_ctx**": "*mut *mut MoeCtx",
    "char*": "*mut c_char", "int*": "*mut i32", "int32_t*": "*mut i32", "float*": "*mut f32",
    "const float*": "*const f32", "uint16_t*": "*mut u16", "const uint16_t*": "*const u16",
    "uint32_t*": "*mut u32", "uint64_t*": "*mut u64", "const uint64_t*": "*const u64",
    "const moe_layer_spec*": "*const MoeLayerSpec", "moe_stage_stat*": "*mut MoeStageStat",
}


def _norm_c_type(decl: str) -> str:
    decl = " ".join(decl.replace("*", " * ").split())
    words = decl.split(" ")
    # drop the parameter name (last identifier) when one is present
    if len(words) > 1 and re.fullmatch(r"[A-Za-z_]\w*", words[-1]) and words[-1] not in C2RUST:
        words = words[:-1]
    t = " ".join(words).replace(" *", "*")
    return t


def header_decls():
    text = (ROOT / "include" / "moe_b200.h").read_text()
    t = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    t = re.sub(r"^\s*#.*$", "", t, flags=re.M)
    out = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(moe_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", t):
        ret = _norm_c_type(m.group(1).strip() + " x")
        params = [p.strip() for p in m.group(3).split(",")]
        args = [] if params == ["void"] else [_norm_c_type(p) for p in params]
        out[m.group(2)] = (ret, args)
    return out


def crate_decls():
    src = (ROOT / "ffi" / "src" / "lib.rs").read_text()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    out = {}
    for m in re.finditer(r"pub fn (moe_[a-z0-9_]+)\s*\((.*?)\)\s*(->\s*([^;]+))?;", block, flags=re.S):
        args = [a.strip() for a in m.group(2).replace("\n", " ").split(",") if a.strip()]
        types = [" ".join(a.split(":", 1)[1].split()) for a in args]
        ret = m.group(4).strip() if m.group(4) else "()"
        assert m.group(1) not in out, f"{m.group(1)} declared twice"
        out[m.group(1)] = (ret, types)
    return out


def test_every_header_function_is_declared_with_matching_types():
    h, r = header_decls(), crate_decls()
    assert sorted(h) == sorted(r), (set(h) ^ set(r))
    for name, (cret, cargs) in h.items():
        rret, rargs = r[name]
        assert C2RUST[cret] == rret, (name, cret, rret)
        assert len(cargs) == len(rargs), (name, cargs, rargs)
        for i, (ca, ra) in enumerate(zip(cargs, rargs)):
            assert C2RUST[ca] == ra, (name, i, ca, ra)


def _c_struct(name):
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "moe_b200.h").read_text(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, text, flags=re.S).group(1)
    fields = []
    for line in body.split(";"):
        line = line.strip()
        if not line:
            continue
        m = re.fullmatch(r"([\w ]+?)\s+(\w+)(\[(\d+)\])?", line)
        fields.append((m.group(2), m.group(1), m.group(4)))
    return fields


def _rust_struct(name):
    src = (ROOT / "ffi" / "src" / "lib.rs").read_text()
    body = re.search(r"#\[repr\(C\)\][^{]*?pub struct %s \{(.*?)\}" % name, src, flags=re.S).group(1)
    return [(m.group(1), m.group(2).strip()) for m in re.finditer(r"pub (\w+):\s*([^,]+),", body)]


def test_repr_c_structs_match_the_header():
    c = _c_struct("moe_layer_spec")
    r = _rust_struct("MoeLayerSpec")
    assert [f for f, _, _ in c] == [f for f, _ in r]
    for (f, ct, _), (_, rt) in zip(c, r):
        assert C2RUST[ct] == rt, (f, ct, rt)
    c = _c_struct("moe_stage_stat")
    r = dict(_rust_struct("MoeStageStat"))
    assert [f for f, _, _ in c] == list(r)
    assert r["name"] == "[c_char; 24]" and r["calls"] == "u32" and r["total_ms"] == "f32"


def test_constants_match_the_header():
    text = (ROOT / "include" / "moe_b200.h").read_text()
    src = (ROOT / "ffi" / "src" / "lib.rs").read_text()
    defs = dict(re.findall(r"#define (MOE_[A-Z0-9_]+) \(?(-?[0-9xA-Fa-f]+)u?\)?", text))
    rust = {n: v.replace("_", "") for n, v in re.findall(r"pub const (MOE_[A-Z0-9_]+): \w+ = (-?[0-9xA-Fa-f_]+);", src)}
    assert set(defs) == set(rust), set(defs) ^ set(rust)
    for n, v in defs.items():
        assert int(v, 0) == int(rust[n], 0), (n, v, rust[n])
