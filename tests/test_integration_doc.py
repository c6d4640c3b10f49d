"""The C# P/Invoke block of INTEGRATION.md against include/aexis_cuda.h: the
same entry points, each DllImport (overloads included) with the header's
argument count. CPU only: the block is parsed as text (there is no .NET here)."""
import os
import re

from aiimage_b200 import native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_arities() -> dict:
    text = re.sub(r"/\*.*?\*/", "", open(native.HEADER).read(), flags=re.S)
    out = {}
    for name, args in re.findall(r"\b(aexis_(?:cuda_|quantize_)\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        args = args.strip()
        out[name] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def csharp_imports() -> list:
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    block = doc[doc.index("```csharp"):]
    block = block[:block.index("```", 3)]
    out = []
    for name, args in re.findall(r"\[DllImport\(Lib\)\]\s*internal static extern \w+\s+(\w+)\s*\(([^;]*?)\)\s*;",
                                 block, flags=re.S):
        args = " ".join(args.split())
        out.append((name, 0 if not args else args.count(",") + 1))
    return out


def test_pinvoke_block_matches_header():
    header = header_arities()
    assert sorted(header) == native.declared_functions()
    imports = csharp_imports()
    names = {n for n, _ in imports}
    assert names == set(header), (sorted(set(header) - names), sorted(names - set(header)))
    wrong = [(n, a, header[n]) for n, a in imports if a != header[n]]
    assert not wrong, wrong


def test_pinvoke_has_fp16_scale_overloads():
    """fp16 scales (scale_dtype AEXIS_F16) need a 16-bit array type on the C# side."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    for name in ("aexis_cuda_weights_q8", "aexis_cuda_weights_q4", "aexis_cuda_decoder_set_linear"):
        assert re.search(name + r"\([^;]*ushort\[\] scales", doc, flags=re.S), name
