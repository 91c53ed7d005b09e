"""A small C prototype reader for the ABI tests: the functions a header declares, with their return and
parameter types normalised (parameter names dropped, whitespace removed), so two headers can be
compared declaration by declaration."""
import re

_BUILTIN = {"void", "char", "short", "int", "long", "float", "double", "signed", "unsigned", "const", "volatile",
            "struct", "enum", "union", "_Float16", "_Bool"}


def _strip(src):
    src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)
    src = re.sub(r"//[^\n]*", " ", src)
    return re.sub(r"^\s*#[^\n]*(\\\n[^\n]*)*", " ", src, flags=re.M)


def _typedefs(src):
    names = set(re.findall(r"typedef\s+[^;{]*?\b(\w+)\s*;", src))
    names |= set(re.findall(r"}\s*(\w+)\s*;", src))  # typedef struct { ... } name;
    return names


def _norm_param(p, types):
    toks = re.findall(r"\w+|\*|\[|\]", p)
    if len(toks) > 1 and re.fullmatch(r"[A-Za-z_]\w*", toks[-1]) and toks[-1] not in _BUILTIN \
            and toks[-1] not in types and not toks[-1].endswith("_t") and toks[-2] != "struct":
        toks = toks[:-1]
    return " ".join(toks).replace(" *", "*").replace("* ", "*")


def prototypes(texts):
    """{name: [return type, [parameter types]]} of every `ork_*` function declared in the given header
    sources (later declarations of a name win)."""
    srcs = [_strip(t) for t in texts]
    types = set()
    for s in srcs:
        types |= _typedefs(s)
    out = {}
    for s in srcs:
        for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(ork_\w+)\s*\(([^;{()]*)\)\s*;", s):
            ret = _norm_param(m.group(1), types | {"x"}).strip()
            params = [x.strip() for x in m.group(3).split(",") if x.strip()]
            out[m.group(2)] = [" ".join(ret.split()), [_norm_param(x, types) for x in params]]
    return out
