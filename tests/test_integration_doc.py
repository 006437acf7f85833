"""The Rust FFI stubs that INTEGRATION.md gives a maintainer name functions the C header
declares, with the same number of parameters (the binding text is not compiled here: the image
has no Rust toolchain, so this is what keeps it from drifting from include/bebelm_attn.h)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _split_params(text: str) -> list:
    text = " ".join(text.split())
    if text.strip() in ("", "void"):
        return []
    return [p for p in (x.strip() for x in text.split(",")) if p]


def _header_functions() -> dict:
    src = open(os.path.join(ROOT, "include", "bebelm_attn.h")).read()
    src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)
    out = {}
    for m in re.finditer(r"BEBELM_API\s+[\w\s\*]+?\b(bebelm_\w+)\s*\(([^;]*?)\)\s*;", src, flags=re.S):
        out[m.group(1)] = len(_split_params(m.group(2)))
    return out


def _rust_stubs() -> dict:
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    out = {}
    for block in re.findall(r"```rust(.*?)```", doc, flags=re.S):
        for m in re.finditer(r"pub fn (bebelm_\w+)\s*\((.*?)\)\s*(?:->|;)", block, flags=re.S):
            out[m.group(1)] = len(_split_params(m.group(2)))
    return out


def test_header_parses():
    h = _header_functions()
    assert len(h) >= 60 and "bebelm_attn_step" in h and h["bebelm_attn_step"] == 14


def test_rust_stubs_match_the_header():
    h, r = _header_functions(), _rust_stubs()
    assert len(r) >= 30, sorted(r)
    missing = sorted(n for n in r if n not in h)
    assert not missing, missing
    wrong = {n: (r[n], h[n]) for n in r if r[n] != h[n]}
    assert not wrong, wrong
