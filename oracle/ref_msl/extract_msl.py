"""Extract the reference's embedded Metal kernel source for the host build.

Reads the Swift multi-line string literal ``let metalSource = \"\"\" ... \"\"\"``
from the reference's full_forward.swift (lines 55-445 of that file) exactly as
it lies, and writes it unchanged to OUT.  Nothing of the reference is copied
into this repository: the output goes to oracle/_ref/ (git-ignored), and this
script only runs where the reference is mounted.

usage: python extract_msl.py <full_forward.swift> <out.metal>
"""
import sys

src, out = sys.argv[1], sys.argv[2]
lines = open(src, encoding="utf-8").read().split("\n")
start = next(i for i, l in enumerate(lines) if l.strip() == 'let metalSource = """')
end = next(i for i in range(start + 1, len(lines)) if lines[i].strip() == '"""')
indent = len(lines[end]) - len(lines[end].lstrip())
body = [l[indent:] for l in lines[start + 1:end]]
text = "\n".join(body) + "\n"
if "\\" in text:
    sys.exit("escape sequences in the Swift literal are not handled; refusing to guess")
with open(out, "w", encoding="utf-8") as f:
    f.write(f"// extracted from {src} lines {start + 2}-{end}\n#line {start + 2} \"{src}\"\n")
    f.write(text)
print(f"extracted {len(body)} lines ({start + 2}-{end}) -> {out}")
