"""CPU: the Rust binding (rust/src/kernel/gdn2_b200.rs) agrees with include/gdn2.h.

The Rust side cannot be compiled here (no Rust toolchain in this image), so
its #[repr(C)] structures are laid out by the C rules in Python and compared,
field by field (name, order, offset) and in total size, with a gcc-compiled
probe of the header; its extern "C" block must declare every entry point the
header declares."""
import os
import re
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn2.h")
RUST = os.path.join(ROOT, "rust", "src", "kernel", "gdn2_b200.rs")
NAMES = {"Gdn2View": "gdn2_view", "Gdn2Dims": "gdn2_dims", "Gdn2ChunkArgs": "gdn2_chunk_args",
         "Gdn2RecurrentArgs": "gdn2_recurrent_args", "Gdn2PrologueArgs": "gdn2_prologue_args",
         "Gdn2Config": "gdn2_config", "Gdn2RecurrentBwdArgs": "gdn2_recurrent_bwd_args"}
PRIM = {"i32": 4, "u32": 4, "f32": 4, "i64": 8, "u64": 8, "f64": 8, "usize": 8}


def rust_structs():
    src = open(RUST).read()
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\]\s*(?:#\[derive\([^)]*\)\]\s*)?pub struct (\w+) \{(.*?)\n\}", src, re.S):
        fields = re.findall(r"pub (\w+): ([^,]+),", m.group(2))
        out[m.group(1)] = [(n, t.strip()) for n, t in fields]
    return out


def rust_layout(structs, name, memo):
    if name in memo:
        return memo[name]
    off, align, fields = 0, 1, []
    for fname, ftype in structs[name]:
        if ftype.startswith("*"):
            size = al = 8
        elif ftype in PRIM:
            size = al = PRIM[ftype]
        else:
            size, al, _ = rust_layout(structs, ftype, memo)
        off = (off + al - 1) // al * al
        fields.append((fname, off))
        off += size
        align = max(align, al)
    size = (off + align - 1) // align * align
    memo[name] = (size, align, fields)
    return memo[name]


def c_structs():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"typedef struct (\w+) \{(.*?)\} \1;", src, re.S):
        names = []
        for decl in m.group(2).split(";"):
            decl = decl.strip()
            if not decl:
                continue
            parts = decl.split(",")
            first = re.match(r"(.*?)([\*\s]*)(\w+)$", parts[0].strip())
            names.append(first.group(3))
            for p in parts[1:]:
                names.append(p.strip().lstrip("*").strip())
        out[m.group(1)] = names
    return out


def c_layout(cs):
    probe = ['#include <stdio.h>', '#include <stddef.h>', '#include "gdn2.h"', "int main() {"]
    for s, fields in cs.items():
        probe.append(f'  printf("{s} size %zu\\n", sizeof({s}));')
        for f in fields:
            probe.append(f'  printf("{s} {f} %zu\\n", offsetof({s}, {f}));')
    probe.append("  return 0;\n}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(src, "w").write("\n".join(probe))
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), src, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {}
    for line in lines:
        if line:
            s, f, v = line.split()
            got[(s, f)] = int(v)
    return got


def test_rust_structs_match_header():
    rs, cs = rust_structs(), c_structs()
    assert set(NAMES.values()) <= set(cs), sorted(cs)
    assert set(NAMES) <= set(rs), sorted(rs)
    offs = c_layout(cs)
    memo = {}
    for rname, cname in NAMES.items():
        size, _, fields = rust_layout(rs, rname, memo)
        assert [f for f, _ in fields] == cs[cname], (rname, [f for f, _ in fields], cs[cname])
        for f, off in fields:
            assert offs[(cname, f)] == off, (rname, f, off, offs[(cname, f)])
        assert offs[(cname, "size")] == size, (rname, size, offs[(cname, "size")])


def test_rust_extern_block_declares_every_entry_point():
    header = set(re.findall(r"GDN2_API\s+[\w\s\*]+?\b(gdn2_\w+)\s*\(", open(HEADER).read()))
    src = open(RUST).read()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}")]
    rust = set(re.findall(r"pub fn (gdn2_\w+)\(", block))
    assert header == rust, (header - rust, rust - header)
    ver = re.search(r"#define GDN2_ABI_VERSION (\d+)", open(HEADER).read()).group(1)
    assert f"pub const GDN2_ABI_VERSION: i32 = {ver};" in src
