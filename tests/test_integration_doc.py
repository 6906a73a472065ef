"""The Rust binding documented for a Chaos maintainer must match the C header.

INTEGRATION.md shows the `-sys` crate a maintainer adds to the reference's Rust workspace. No
Rust toolchain exists here, so nothing compiles it; instead this test parses the header
(`include/bigtea_decode.h`) and the documented `extern "C"` block and checks, item by item:

- every constant (`BT_ABI_VERSION`, the status codes, type ids, policies) has the header's value;
- every `#[repr(C)]` struct has the header struct's fields, in order, with the mapped types;
- every header function is declared with the same parameter and return types, and nothing else
  is declared.

A struct that drifted (a missing field would make `bt_engine_create` read past the caller's
struct) or a stale ABI version fails here.
"""
import os
import re

from bigtea_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bigtea_decode.h")
DOC = os.path.join(ROOT, "INTEGRATION.md")

C_BASE = {"uint32_t": "u32", "uint64_t": "u64", "int32_t": "i32", "int8_t": "i8", "uint8_t": "u8", "int": "c_int",
          "float": "f32", "double": "f64", "size_t": "usize", "char": "c_char", "void": "c_void"}


def _strip_c_comments(text):
    return re.sub(r"/\*.*?\*/", "", text, flags=re.S)


def c_to_rust(ctype: str) -> str:
    """A C parameter/field type as the Rust FFI spells it (`const T *` -> `*const T`)."""
    t = ctype.replace("*", " * ").split()
    const_pointee = "const" in t[:t.index("*")] if "*" in t else False
    words = [w for w in t if w not in ("const", "*")]
    assert len(words) == 1, ctype
    base = C_BASE.get(words[0], words[0])
    n = t.count("*")
    if n == 0:
        return base
    out = ("*const " if const_pointee else "*mut ") + base
    for _ in range(n - 1):
        out = "*mut " + out
    return out


def _split_decl(decl: str):
    """'const uint32_t *seq_ids' -> ('const uint32_t *', 'seq_ids')"""
    decl = decl.strip()
    m = re.match(r"^(.*?)(\w+)\s*$", decl)
    return m.group(1).strip(), m.group(2)


def parse_header():
    text = open(HEADER).read()
    consts = {}
    for name, expr in re.findall(r"#define\s+(BT_\w+)\s+([^\n]+)", text):
        expr = re.sub(r"(\d+)[uU]", r"\1", expr.split("/*")[0]).strip()
        if re.fullmatch(r"[\d\s()<>|+*]+", expr):  # integer literals and shifts only
            consts[name] = int(eval(expr))
    body = _strip_c_comments(text)
    for block in re.findall(r"enum\s*\{(.*?)\}", body, flags=re.S):
        for name, val in re.findall(r"(BT_\w+)\s*=\s*(\d+)", block):
            consts[name] = int(val)
    structs = {}
    for inner, name in re.findall(r"typedef\s+struct\s*\w*\s*\{(.*?)\}\s*(\w+)\s*;", body, flags=re.S):
        fields = []
        for stmt in inner.split(";"):
            stmt = " ".join(stmt.split())
            if not stmt:
                continue
            first, *rest = stmt.split(",")
            ty, f0 = _split_decl(re.sub(r"\[\d+\]", "", first))
            arr0 = re.search(r"\[(\d+)\]", first)
            decls = [(f0, arr0.group(1) if arr0 else None)]
            for r in rest:
                arr = re.search(r"\[(\d+)\]", r)
                decls.append((re.sub(r"[\[\]\d\s\*]", "", r) if arr else r.strip(), arr.group(1) if arr else None))
            for fname, arr in decls:
                rt = c_to_rust(ty)
                fields.append((fname, f"[{rt}; {arr}]" if arr else rt))
        structs[name] = fields
    funcs = {}
    flat = " ".join(re.sub(r"^\s*#.*$", "", body, flags=re.M).split())
    for ret, name, params in re.findall(r"([\w\s\*]+?)\b(bt_\w+)\s*\(([^()]*)\)\s*;", flat):
        ret = ret.strip().split()
        ret = " ".join(w for w in ret if w not in ("typedef",))
        plist = [] if params.strip() in ("", "void") else [c_to_rust(_split_decl(p)[0]) for p in params.split(",")]
        r = None if ret == "void" else c_to_rust(ret)
        funcs[name] = (plist, r)
    return consts, structs, funcs


def rust_block():
    md = open(DOC).read()
    blocks = re.findall(r"```rust\n(.*?)```", md, flags=re.S)
    ext = [b for b in blocks if 'extern "C"' in b]
    assert len(ext) == 1, "INTEGRATION.md must hold exactly one Rust block with the extern \"C\" declarations"
    return ext[0]


def parse_rust(code: str):
    code = re.sub(r"//[^\n]*", "", code)
    consts = {n: int(v) for n, v in re.findall(r"pub\s+const\s+(\w+)\s*:\s*\w+\s*=\s*(\d+)\s*;", code)}
    structs = {}
    for name, inner in re.findall(r"#\[repr\(C\)\]\s*pub\s+struct\s+(\w+)\s*\{(.*?)\}", code, flags=re.S):
        fields = []
        for f, ty in re.findall(r"pub\s+(\w+)\s*:\s*([^,]+?)\s*(?:,|$)", " ".join(inner.split())):
            fields.append((f[:-1] if f.endswith("_") else f, " ".join(ty.split())))
        structs[name] = fields
    funcs = {}
    ext = code[code.index('extern "C"'):]
    for name, params, ret in re.findall(r"pub\s+fn\s+(\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+))?;", ext, flags=re.S):
        plist = [" ".join(p.split(":", 1)[1].split()) for p in params.split(",") if p.strip()]
        funcs[name] = (plist, " ".join(ret.split()) if ret else None)
    return consts, structs, funcs


def test_c_to_rust_mapping():
    assert c_to_rust("const uint32_t *") == "*const u32"
    assert c_to_rust("bt_engine **") == "*mut *mut bt_engine"
    assert c_to_rust("void *") == "*mut c_void"
    assert c_to_rust("const char *") == "*const c_char"
    assert c_to_rust("size_t") == "usize"


def test_documented_constants_match_the_header():
    hc, _, _ = parse_header()
    rc, _, _ = parse_rust(rust_block())
    assert hc["BT_ABI_VERSION"] == _lib.ABI_VERSION
    for name in ("BT_ABI_VERSION", "BT_OK", "BT_ERR_INVALID", "BT_ERR_CUDA", "BT_ERR_OOM", "BT_ERR_MISSING_TENSOR",
                 "BT_ERR_KV", "BT_ERR_TIMEOUT", "BT_ERR_UNSUPPORTED", "BT_KV_F16", "BT_XCACHE_LRU",
                 "BT_XCACHE_FREQ"):
        assert name in rc, f"{name} is not documented"
    for name, val in rc.items():
        assert hc.get(name) == val, f"{name}: documented {val}, header {hc.get(name)}"


def test_documented_structs_match_the_header():
    _, hs, _ = parse_header()
    _, rs, _ = parse_rust(rust_block())
    for name in ("bt_model_desc", "bt_tensor_view", "bt_stats", "bt_kernel_time", "bt_xcache_stats",
                 "bt_sampler_config", "bt_sampler_state"):
        assert name in rs, f"struct {name} is not documented"
        assert rs[name] == hs[name], f"struct {name}: documented {rs[name]}, header {hs[name]}"


def test_documented_functions_match_the_header():
    _, _, hf = parse_header()
    _, _, rf = parse_rust(rust_block())
    assert len(hf) >= 35
    assert set(rf) == set(hf), (sorted(set(hf) - set(rf)), sorted(set(rf) - set(hf)))
    for name, (params, ret) in hf.items():
        assert rf[name] == (params, ret), f"{name}: documented {rf[name]}, header {(params, ret)}"
    # the ctypes mirror declares the same functions with the same arity
    for name, (params, _) in hf.items():
        assert len(_lib.SIGNATURES[name][1]) == len(params), name
