"""The Rust FFI crate (rust/scratchtape-b200-sys) against include/st_b200.h,
on CPU: there is no Rust toolchain in this image, so the crate is checked by
reading it.  Every ST_API function must appear in the extern block with the
same parameter list (types mapped C -> Rust) and return type, and nothing
else may; the repr(C) structs must list the header's fields in order with
the same types; the status codes must have the header's values."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "st_b200.h")
LIB = os.path.join(ROOT, "rust", "scratchtape-b200-sys", "src", "lib.rs")

C2R = {"int64_t": "i64", "int32_t": "i32", "int": "c_int", "uint32_t": "u32", "uint64_t": "u64", "float": "f32",
       "st_status": "st_status", "st_precision": "c_int", "uint8_t": "u8", "void": "c_void", "char": "c_char",
       "st_handle": "st_handle", "st_mat": "st_mat", "st_epilogue": "st_epilogue", "st_group_gemm": "st_group_gemm"}


def _rust_of(c):
    c = " ".join(c.split())
    const = c.startswith("const ")
    if const:
        c = c[6:]
    stars = c.count("*")
    base = C2R[c.replace("*", "").strip()]
    if stars == 0:
        return base
    if stars == 1:
        return ("*const " if const else "*mut ") + base
    return "*mut " * stars + base


def _header_functions():
    src = re.sub(r"/\*.*?\*/", "", open(HDR).read(), flags=re.S)
    out = {}
    for d in re.findall(r"^ST_API\s+(.*?);", src, flags=re.S | re.M):
        d = " ".join(d.split())
        m = re.match(r"(.*?)\b(st_\w+)\s*\((.*)\)$", d)
        args = []
        for a in m.group(3).split(","):
            am = re.match(r"(.*?)(\w+)$", a.strip())
            args.append(_rust_of(am.group(1)))
        out[m.group(2)] = (_rust_of(m.group(1)), args)
    return out


def _rust_functions():
    src = open(LIB).read()
    block = re.search(r'extern "C" \{(.*?)\n\}', src, flags=re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (st_\w+)\((.*?)\)\s*->\s*([^;]+);", block, flags=re.S):
        args = [" ".join(a.split(":", 1)[1].split()) for a in m.group(2).split(",") if a.strip()]
        out[m.group(1)] = (" ".join(m.group(3).split()), args)
    return out


def test_extern_block_matches_every_header_declaration():
    want, got = _header_functions(), _rust_functions()
    assert len(want) >= 40
    assert sorted(got) == sorted(want), "extern block and header list different functions: %s" % (
        sorted(set(got) ^ set(want)))
    for name, (ret, args) in want.items():
        assert got[name][0] == ret, "%s returns %s in the crate, %s in the header" % (name, got[name][0], ret)
        assert got[name][1] == args, "%s parameters differ:\n crate  %s\n header %s" % (name, got[name][1], args)


def _header_struct(name):
    src = re.sub(r"/\*.*?\*/", "", open(HDR).read(), flags=re.S)
    body = re.search(r"typedef struct \{([^}]*)\}\s*%s;" % name, src, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        m = re.match(r"(.*?)([\w\s,]+)$", decl)
        ty = m.group(1).strip()
        names = [n.strip() for n in m.group(2).split(",")]
        if not ty:  # "st_mat a, b, out": the type is the first word
            first, rest = names[0].split(" ", 1)
            ty, names = first, [rest] + names[1:]
        for n in names:
            stars = n.count("*")
            fields.append((n.replace("*", "").strip(), _rust_of(ty + "*" * stars)))
    return fields


def _rust_struct(name):
    src = open(LIB).read()
    body = re.search(r"pub struct %s \{(.*?)\}" % name, src, flags=re.S).group(1)
    return [(n.strip().replace("pub ", ""), " ".join(t.split())) for n, t in
            (f.split(":", 1) for f in body.split(",") if f.strip())]


def test_structs_match_the_header():
    for name in ("st_mat", "st_epilogue", "st_group_gemm"):
        assert _rust_struct(name) == _header_struct(name), name


def test_status_codes_match_the_header():
    hdr = open(HDR).read()
    want = dict((k, int(v)) for k, v in re.findall(r"(ST_[A-Z_]+) = (\d+)", hdr))
    got = dict((k, int(v)) for k, v in re.findall(r"pub const (ST_[A-Z_0-9]+): st_status = (\d+);", open(LIB).read()))
    assert got and all(want[k] == v for k, v in got.items())
    assert set(got) == {k for k in want if k in ("ST_OK", "ST_INVALID_ARG", "ST_UNSUPPORTED_SHAPE", "ST_CUDA_ERROR",
                                                 "ST_NCCL_ERROR", "ST_TIMEOUT", "ST_NO_MEMORY", "ST_NOT_FOUND")}
