"""The Rust binding (whisper.rs_b200/rust/whisper-attn-cuda) against the C ABI.

No Rust toolchain is available here, so the crate is checked as text: its
`extern "C"` block must declare exactly the entry points of include/wattn.h,
each with the same parameter and return types (C types mapped to their Rust
FFI spellings), the Python host module must bind the same arities, and
build.rs must compile every CUDA source of the library.
"""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "wattn.h")
CRATE = os.path.join(ROOT, "whisper.rs_b200", "rust", "whisper-attn-cuda")
CSRC = os.path.join(ROOT, "whisper.rs_b200", "csrc")

C_TO_RUST = {
    "int": "c_int", "int64_t": "i64", "size_t": "usize", "float": "f32", "void": "()",
    "void*": "*mut c_void", "const void*": "*const c_void",
    "float*": "*mut f32", "const float*": "*const f32",
    "int*": "*mut c_int", "const int*": "*const c_int",
    "char*": "*mut c_char", "const char*": "*const c_char",
    "wattn_kv_cache*": "*mut wattn_kv_cache", "const wattn_kv_cache*": "*const wattn_kv_cache",
    "wattn_kv_cache**": "*mut *mut wattn_kv_cache",
}


def _c_type(decl: str) -> str:
    """'const void *q' -> 'const void*' (the parameter name dropped)."""
    decl = " ".join(decl.replace("*", " * ").split())
    toks = decl.split(" ")
    if toks[-1] not in ("*", "void") and len(toks) > 1:
        toks = toks[:-1]  # the name
    return re.sub(r"\s*\*", "*", " ".join(toks)).strip()


def header_decls():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, params in re.findall(
            r"((?:const\s+)?[a-z_0-9]+\s*\**)\s*(wattn_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        ps = [] if params.strip() in ("", "void") else [_c_type(p) for p in params.split(",")]
        out[name] = (_c_type(ret + " x"), ps)
    return out


def rust_decls():
    src = open(os.path.join(CRATE, "src", "lib.rs")).read()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    out = {}
    for name, params, ret in re.findall(
            r"pub fn (wattn_[a-z0-9_]+)\(([^)]*)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        ps = [p.split(":", 1)[1].strip() for p in params.split(",") if p.strip()]
        out[name] = ((ret or "()").strip(), [" ".join(p.split()) for p in ps])
    return out


def test_header_parses():
    decls = header_decls()
    assert "wattn_attention_fwd" in decls and len(decls["wattn_attention_fwd"][1]) == 21
    assert decls["wattn_version"] == ("int", [])
    assert decls["wattn_status_string"][0] == "const char*"


def test_rust_extern_block_matches_the_header():
    h, r = header_decls(), rust_decls()
    assert sorted(r) == sorted(h), (set(h) ^ set(r))
    for name, (ret, params) in h.items():
        rret, rparams = r[name]
        assert C_TO_RUST[ret] == rret, f"{name}: return {ret} vs {rret}"
        assert [C_TO_RUST[p] for p in params] == rparams, f"{name}: {params} vs {rparams}"


def test_python_binding_matches_the_header():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "whisper.rs_b200"))
    import wattn
    h = header_decls()
    assert sorted(wattn._SIGS) == sorted(h)
    for name, (_, params) in h.items():
        assert len(wattn._SIGS[name][1]) == len(params), name


def test_build_rs_compiles_every_cuda_source():
    text = open(os.path.join(CRATE, "build.rs")).read()
    m = re.search(r"const SOURCES: \[&str; (\d+)\] = \[(.*?)\];", text, flags=re.S)
    assert m, "SOURCES list not found"
    listed = re.findall(r'"([a-z0-9_]+)"', m.group(2))
    assert int(m.group(1)) == len(listed)
    on_disk = sorted(f[:-3] for f in os.listdir(CSRC) if f.endswith(".cu"))
    assert sorted(listed) == on_disk


def test_device_kv_cache_mirrors_decoder_kv_cache():
    """Every public method of DecoderKvCache (crates/whisper/src/decoder.rs:
    147-264) has its namesake on DeviceKvCache, plus the per-layer steps."""
    src = open(os.path.join(CRATE, "src", "lib.rs")).read()
    impl = src[src.index("impl DeviceKvCache {"):src.index("impl Drop for DeviceKvCache")]
    methods = set(re.findall(r"pub (?:unsafe )?fn ([a-z_]+)\(", impl))
    reference = {"new", "clear", "clear_slot", "invalidate_cross", "ensure_slots", "copy_slot",
                 "slot_len", "slide_to_fit"}
    steps = {"append", "attend", "advance", "set_t_past", "assign_beams"}
    missing = (reference | steps) - methods
    assert not missing, missing


@pytest.mark.parametrize("fn", ["flash_attention_2", "multi_head_attention",
                                "single_token_mha_d64", "multi_head_attention_with_cache",
                                "capture_cross_attention_heads"])
def test_reference_signatures_kept(fn):
    src = open(os.path.join(CRATE, "src", "lib.rs")).read()
    i = src.index("pub fn " + fn + "(") + len("pub fn " + fn + "(")
    depth, params, cur = 0, [], ""
    for ch in src[i:]:  # the parameter list, split at top-level commas
        if ch in "([":
            depth += 1
        elif ch in ")]":
            if depth == 0:
                break
            depth -= 1
        if ch == "," and depth == 0:
            params.append(cur)
            cur = ""
        else:
            cur += ch
    params.append(cur)
    names = [p.split(":")[0].strip() for p in params if p.strip()]
    expected = {
        "flash_attention_2": ["q", "k", "v", "t_q", "t_kv", "n_heads", "d_model", "causal",
                              "output"],
        "multi_head_attention": ["q", "k", "v", "t_q", "t_kv", "n_heads", "d_model", "causal",
                                 "output"],
        "single_token_mha_d64": ["q", "k", "v", "t_kv", "n_heads", "d_model", "output"],
        "multi_head_attention_with_cache": ["q", "k", "v", "n_tokens", "total_tokens", "t_past",
                                            "n_heads", "d_model", "output"],
        "capture_cross_attention_heads": ["q", "k", "n_tokens", "n_audio", "n_heads", "d_model",
                                          "selected", "n_selected", "row_offset", "out"],
    }[fn]
    assert names == expected
