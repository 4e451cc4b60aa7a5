"""The Rust crate qora-cuda-sys (qora-llm_b200/rust/qora-cuda-sys) against the C ABI it
binds. There is no Rust toolchain on this machine, so the crate is checked here without
compiling it: every function, struct and constant of include/qora_cuda.h must appear in
the crate's raw bindings with the same name, the same parameter and field types in the
same order (mapped C -> Rust: uint32_t -> u32, const T* -> *const T, T** -> *mut *mut T,
void* -> *mut c_void, ...) and the same value; and the safe layer must offer the
reference's entry points by name."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qora_cuda.h")
CRATE = os.path.join(ROOT, "qora-llm_b200", "rust", "qora-cuda-sys")

BASE = {"uint8_t": "u8", "uint16_t": "u16", "uint32_t": "u32", "uint64_t": "u64", "int32_t": "i32",
        "int": "c_int", "size_t": "usize", "float": "f32", "char": "c_char", "void": "c_void",
        "qora_status": "qora_status"}


def _read(path):
    with open(path) as f:
        return f.read()


def _strip_c(src):
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.sub(r"//[^\n]*", "", src)


def _strip_rs(src):
    return re.sub(r"//[^\n]*", "", src)


def c_to_rust(t):
    """'const uint8_t*' -> '*const u8', 'qora_kv**' -> '*mut *mut qora_kv'."""
    t = " ".join(t.replace("*", " * ").split())
    const = t.startswith("const ")
    if const:
        t = t[len("const "):]
    stars = t.count("*")
    base = t.replace("*", "").strip()
    base = BASE.get(base, base)
    if stars == 0:
        return base
    if stars == 1:
        return ("*const " if const else "*mut ") + base
    return "*mut " * stars + base  # double pointers are the non-const out-parameters


def _norm_rs(t):
    return " ".join(t.replace("*", " *").split()).replace("* ", "*")


def header_functions():
    src = _strip_c(_read(HEADER))
    out = {}
    for ret, name, params in re.findall(r"(qora_status|void|const char\s*\*)\s+(qora_\w+)\s*\(([^)]*)\)\s*;", src):
        ps = []
        if params.strip() not in ("", "void"):
            for p in params.split(","):
                p = " ".join(p.split())
                ty = re.sub(r"\s*\b\w+$", "", p)  # drop the parameter name
                ps.append(c_to_rust(ty))
        r = None if ret == "void" else c_to_rust(" ".join(ret.split()))
        out[name] = (r, ps)
    return out


def crate_functions():
    src = _strip_rs(_read(os.path.join(CRATE, "src", "lib.rs")))
    block = re.search(r'extern "C" \{(.*)\n\}', src, flags=re.S).group(1)
    out = {}
    for name, params, ret in re.findall(r"pub fn (\w+)\(([^)]*)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        ps = [_norm_rs(p.split(":", 1)[1]) for p in params.split(",") if p.strip()]
        out[name] = (_norm_rs(ret) if ret else None, ps)
    return out


def header_structs():
    src = _strip_c(_read(HEADER))
    out = {}
    for body, name in re.findall(r"typedef struct \w+ \{(.*?)\}\s*(\w+)\s*;", src, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            m = re.match(r"^((?:const )?\w+\s*\**)\s*(.+)$", decl)
            ty, names = m.group(1), m.group(2)
            for n in names.split(","):
                fields.append((n.strip(), c_to_rust(ty)))
        out[name] = fields
    return out


def crate_structs():
    src = _strip_rs(_read(os.path.join(CRATE, "src", "lib.rs")))
    out = {}
    for name, body in re.findall(r"pub struct (\w+) \{(.*?)\}", src, flags=re.S):
        out[name] = [(n, _norm_rs(t)) for n, t in re.findall(r"pub (\w+): ([^,]+),", body)]
    return out


def _eval(expr):
    return eval(re.sub(r"(\d+)u\b", r"\1", expr), {"__builtins__": {}})


def header_constants():
    src = _strip_c(_read(HEADER))
    return {n: _eval(v) for n, v in re.findall(r"#define (QORA_\w+)\s+(.+)", src) if n != "QORA_CUDA_H"}


def crate_constants():
    src = _strip_rs(_read(os.path.join(CRATE, "src", "lib.rs")))
    return {n: _eval(v) for n, v in re.findall(r"pub const (QORA_\w+): \w+ = ([^;]+);", src)}


def test_type_mapping():
    assert c_to_rust("const uint8_t*") == "*const u8"
    assert c_to_rust("qora_kv**") == "*mut *mut qora_kv"
    assert c_to_rust("void*") == "*mut c_void"
    assert c_to_rust("const void*") == "*const c_void"
    assert c_to_rust("const char*") == "*const c_char"
    assert c_to_rust("size_t") == "usize"


def test_every_function_is_bound_with_its_signature():
    import test_abi  # the ABI test's own parser of the header finds the same functions
    h, r = header_functions(), crate_functions()
    assert set(h) == set(test_abi.declared_functions())
    assert sorted(h) == sorted(r), (set(h) ^ set(r))
    for name, sig in h.items():
        assert r[name] == sig, (name, sig, r[name])


def test_every_struct_has_the_same_fields():
    h, r = header_structs(), crate_structs()
    assert set(h) == {"qora_matrix_view", "qora_layer_view", "qora_weights_view", "qora_engine_options",
                      "qora_tp_shard", "qora_sampling"}
    for name, fields in h.items():
        assert r[name] == fields, name
    assert "qora_engine" in r and "qora_kv" in r  # opaque handles


def test_every_constant_has_the_same_value():
    h, r = header_constants(), crate_constants()
    assert h and h == r, (set(h) ^ set(r))


@pytest.mark.parametrize("name", ["load_model", "empty_kv_cache", "forward_decode_raw", "raw_prefill",
                                  "try_forward_decode_raw", "try_raw_prefill", "generate_greedy", "greedy",
                                  "sample_next", "decode_greedy", "tp_plan"])
def test_safe_layer_offers_the_reference_entry_points(name):
    src = _read(os.path.join(CRATE, "src", "safe.rs"))
    assert re.search(rf"pub (?:unsafe )?fn {name}\b", src), name


def test_crate_manifest_links_the_library():
    toml = _read(os.path.join(CRATE, "Cargo.toml"))
    assert 'name = "qora-cuda-sys"' in toml and 'links = "qora_cuda"' in toml
    build = _read(os.path.join(CRATE, "build.rs"))
    assert "rustc-link-lib=dylib=qora_cuda" in build
