"""The Mojo binding stubs of the repository's integration guide cannot be
compiled here (no Mojo toolchain), so this keeps them exact by reading them
as text: every
`get_function[fn (...) -> R]("ms_...")` names a function the header
declares, with the same number of arguments and the same kind of value in
each place (pointer, 32-bit integer, 32-bit float, 64-bit integer), and the
same kind of return value."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def split_top(s):
    """Split on commas outside brackets / parentheses."""
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch in "[(":
            depth += 1
        elif ch in "])":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur)
            cur = ""
        else:
            cur += ch
    out.append(cur)
    return [x.strip() for x in out if x.strip()]


def c_kind(decl):
    """Kind of a C parameter or return type."""
    if "*" in decl:
        return "ptr"
    t = re.sub(r"\b(const|MS_API)\b", "", decl).split()
    base = " ".join(t[:-1]) if len(t) > 1 and not decl.strip().endswith(
        ("int", "float", "size_t", "uint64_t", "ms_status", "void", "double")) else " ".join(t)
    base = base.strip()
    if base in ("int", "ms_status", "int32_t"):
        return "i32"
    if base == "float":
        return "f32"
    if base in ("uint64_t", "size_t", "int64_t"):
        return "i64"
    if base == "double":
        return "f64"
    if base == "void":
        return "void"
    return "?" + base


def mojo_kind(t):
    t = t.strip()
    if t in ("Int32", "UInt32"):
        return "i32"
    if t == "Float32":
        return "f32"
    if t in ("UInt64", "Int64", "Int", "UInt"):
        return "i64"
    if t == "Float64":
        return "f64"
    if t in ("NoneType", "None"):
        return "void"
    return "ptr"  # UnsafePointer[...] and the handle aliases (Ctx, Model, KV, ...)


def header_prototypes():
    hdr = open(os.path.join(ROOT, "include", "mojostream_cuda.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    protos = {}
    for m in re.finditer(r"MS_API\s+([\w\s\*]+?)\s*\b(ms_\w+)\s*\(([^;]*?)\)\s*;", hdr, flags=re.S):
        ret = m.group(1).strip()
        args = m.group(3).strip()
        params = [] if args in ("", "void") else split_top(args)
        protos[m.group(2)] = (c_kind(ret), [c_kind(p) for p in params])
    return protos


def mojo_stubs():
    md = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    pat = r'get_function\[\s*fn\s*\((.*?)\)\s*->\s*(.+?)\]\s*\(\s*"(ms_\w+)"\s*\)'
    return [(m.group(3), [mojo_kind(a) for a in split_top(m.group(1))], mojo_kind(m.group(2)))
            for m in re.finditer(pat, md, flags=re.S)]


def test_header_parses():
    protos = header_prototypes()
    assert len(protos) >= 40
    assert protos["ms_init"] == ("i32", ["i32", "ptr"])
    assert all(not k.startswith("?") for r, a in protos.values() for k in [r] + a), protos


def test_mojo_stubs_match_the_header():
    protos = header_prototypes()
    stubs = mojo_stubs()
    assert len(stubs) >= 10, stubs
    for name, args, ret in stubs:
        assert name in protos, f"{name}: not declared in the header"
        c_ret, c_args = protos[name]
        assert len(args) == len(c_args), f"{name}: {len(args)} arguments, header {len(c_args)}"
        assert args == c_args, f"{name}: argument kinds {args}, header {c_args}"
        assert ret == c_ret, f"{name}: returns {ret}, header {c_ret}"
