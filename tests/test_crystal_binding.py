"""The Crystal `lib GSCuda` binding (crystal-gausplat_b200/crystal/gsplat_cuda.cr)
against include/gsplat_cuda.h, without a Crystal compiler: every C entry
point has exactly one `fun` with the same symbol, argument count and argument
and return types (C types mapped to Crystal's), every struct has the same
fields in the same order with the same types, and every constant has the
header's value. This is the check a maintainer of the reference's Crystal host
relies on when the binding replaces the Metal FFI blocks for this path
(src/gaussian_splatting/rasterizer.cr:28-45, src/metal/gpu_radix_sort.cr:26-40)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gsplat_cuda.h")
BINDING = os.path.join(ROOT, "crystal-gausplat_b200", "crystal", "gsplat_cuda.cr")

SCALARS = {"int": "Int32", "int32_t": "Int32", "int64_t": "Int64", "uint64_t": "UInt64",
           "uint32_t": "UInt32", "uint8_t": "UInt8", "char": "UInt8", "float": "Float32",
           "double": "Float64", "size_t": "LibC::SizeT", "void": "Void"}
STRUCTS = {"gsc_camera": "Camera", "gsc_raster_config": "RasterConfig", "gsc_gaussians": "Gaussians",
           "gsc_gaussian_grads": "GaussianGrads", "gsc_projected": "Projected",
           "gsc_grads2d": "Grads2D", "gsc_adam_group": "AdamGroup",
           "gsc_dp_adam_args": "DpAdamArgs", "gsc_gaussians_out": "GaussiansOut",
           "gsc_dp_barrier_args": "DpBarrierArgs"}
OPAQUE = {"gsc_ctx": "Ctx", "gsc_frame": "Frame"}  # Crystal `type X = Void*`


def _strip_c(src):
    return re.sub(r"/\*.*?\*/", "", src, flags=re.S)


def c_type(decl):
    """Crystal spelling of a C type such as 'const gsc_frame* const*'."""
    t = decl.replace("const", " ")
    stars = t.count("*")
    base = t.replace("*", " ").split()
    assert len(base) == 1, decl
    base = base[0]
    if base in OPAQUE:
        assert stars >= 1, decl
        return OPAQUE[base] + "*" * (stars - 1)
    name = SCALARS.get(base) or STRUCTS.get(base)
    assert name, f"unmapped C type {decl!r}"
    return name + "*" * stars


def header_functions():
    src = _strip_c(open(HEADER).read())
    out = {}
    for m in re.finditer(r"GSC_API\s+([\w\s\*]+?)\b(gsc_\w+)\s*\(([^)]*)\)\s*;", src):
        ret, name, args = m.group(1), m.group(2), " ".join(m.group(3).split())
        types = []
        if args != "void":
            for a in args.split(","):
                a = a.strip()
                pname = re.search(r"(\w+)$", a).group(1)
                types.append(c_type(a[: len(a) - len(pname)]))
        out[name] = (c_type(ret), types)
    return out


def header_structs():
    src = _strip_c(open(HEADER).read())
    out = {}
    for m in re.finditer(r"typedef struct (gsc_\w+) \{(.*?)\} \1;", src, flags=re.S):
        fields = []
        for line in m.group(2).split(";"):
            line = " ".join(line.split())
            if not line:
                continue
            mm = re.match(r"((?:const )?[\w]+\s*\**)\s*(.+)$", line)
            base, names = mm.group(1), mm.group(2)
            for nm in names.split(","):
                nm = nm.strip()
                stars = nm.count("*")
                nm = nm.replace("*", "").strip()
                arr = re.match(r"(\w+)\[(\w+)\]", nm)
                t = c_type(base + "*" * stars)
                if arr:
                    n = arr.group(2)
                    n = str(header_defines().get(n, n))
                    fields.append((arr.group(1), f"StaticArray({t}, {n})"))
                else:
                    fields.append((nm, t))
        out[STRUCTS[m.group(1)]] = fields
    return out


def header_defines():
    src = _strip_c(open(HEADER).read())
    out = {}
    for m in re.finditer(r"#define GSC_(\w+) \(?(-?\d+)u?\)?", src):
        out["GSC_" + m.group(1)] = int(m.group(2))
    return out


def binding_text():
    return re.sub(r"#[^\n]*", "", open(BINDING).read())  # drop comments


def binding_functions():
    src = binding_text()
    out = {}
    for m in re.finditer(r"\bfun\s+(\w+)\s*=\s*(gsc_\w+)\s*(\((.*?)\))?\s*:\s*([\w:\*]+)", src, flags=re.S):
        args = m.group(4)
        types = []
        if args and args.strip():
            for a in " ".join(args.split()).split(","):
                pname, t = [x.strip() for x in a.split(":", 1)]
                types.append(t.replace(" ", ""))
        assert m.group(2) not in out, f"{m.group(2)} bound twice"
        out[m.group(2)] = (m.group(5), types)
    return out


def binding_structs():
    src = binding_text()
    out = {}
    for m in re.finditer(r"\bstruct\s+(\w+)\s*\n(.*?)\n\s*end\b", src, flags=re.S):
        fields = []
        for line in m.group(2).split("\n"):
            line = line.strip()
            if line:
                name, t = [x.strip() for x in line.split(":", 1)]
                fields.append((name, t.replace(" ", "").replace(",", ", ")))
        out[m.group(1)] = fields
    return out


def test_every_header_function_is_bound_with_the_same_signature():
    h, b = header_functions(), binding_functions()
    assert len(h) >= 40
    assert sorted(b) == sorted(h), (set(h) ^ set(b))
    for name, (ret, args) in h.items():
        bret, bargs = b[name]
        assert bret == ret, f"{name}: return {bret} != {ret}"
        assert len(bargs) == len(args), f"{name}: {len(bargs)} arguments, header has {len(args)}"
        for i, (x, y) in enumerate(zip(bargs, args)):
            assert x == y, f"{name} argument {i}: {x} != {y}"


def test_every_struct_has_the_header_fields():
    h, b = header_structs(), binding_structs()
    assert sorted(b) == sorted(h)
    norm = lambda s: s.lstrip("_").lower()  # noqa: E731 (`_pad` -> `pad`, `final_T` -> `final_t`)
    for name, fields in h.items():
        got = [(norm(n), t) for n, t in b[name]]
        want = [(norm(n), t) for n, t in fields]
        assert got == want, name


def test_constants_match_the_header():
    defs = header_defines()
    src = binding_text()
    consts = {m.group(1): int(m.group(2).replace("_u32", "").replace("_", ""))
              for m in re.finditer(r"^\s*([A-Z][A-Z0-9_]+)\s*=\s*(-?[\d_]+(?:_u32)?)\s*$", src, flags=re.M)}
    assert len(consts) >= 25
    for k, v in consts.items():
        assert defs["GSC_" + k] == v, k


def test_camera_is_packed_like_the_reference():
    src = binding_text()
    assert re.search(r"@\[Packed\]\s*struct Camera\b", src)
