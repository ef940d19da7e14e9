"""Rewrites one CUDA source file so that g++ compiles it against the SIMT
emulation headers in this directory.  TEST INFRASTRUCTURE ONLY: it runs at
build time on the reference's own sources (read where they lie) and writes the
result under oracle/_ref/, which is never committed.

Two constructs have no C++ spelling and are rewritten; everything else is left
as it is:

* ``K<<<grid, block[, smem[, stream]]>>>(args);`` becomes
  ``::rpgemu::Launch(dim3(grid), dim3(block), smem, stream, &K, args);``
* ``extern __shared__ T name[];`` becomes a pointer to the block's dynamic
  shared memory, ``T* name = reinterpret_cast<T*>(::rpgemu::DynSmem());``

A ``#line`` directive keeps compiler messages pointing at the original file.

    python prep_cu.py <in.cu> <out.cc>
"""

import re
import sys


def _match_forward(s, i, open_c, close_c):
    """Index of the bracket closing the one at s[i]."""
    depth = 0
    for j in range(i, len(s)):
        if s[j] == open_c:
            depth += 1
        elif s[j] == close_c:
            depth -= 1
            if depth == 0:
                return j
    raise ValueError(f"unbalanced {open_c!r} at offset {i}")


def _split_top(s):
    parts, depth, cur = [], 0, []
    for c in s:
        if c in "([{":
            depth += 1
        elif c in ")]}":
            depth -= 1
        if c == "," and depth == 0:
            parts.append("".join(cur).strip())
            cur = []
        else:
            cur.append(c)
    if "".join(cur).strip():
        parts.append("".join(cur).strip())
    return parts


def _kernel_name_start(s, j):
    """Start of the kernel expression that ends right before s[j] ('<<<')."""
    k = j
    while k > 0 and s[k - 1].isspace():
        k -= 1
    if s[k - 1] == ">":  # template arguments
        depth = 0
        while True:
            k -= 1
            if s[k] == ">":
                depth += 1
            elif s[k] == "<":
                depth -= 1
                if depth == 0:
                    break
    while k > 0 and (s[k - 1].isalnum() or s[k - 1] in "_:"):
        k -= 1
    return k


def rewrite(src: str) -> str:
    src = re.sub(r"extern\s+__shared__\s+([\w:]+)\s+(\w+)\s*\[\s*\]\s*;",
                 r"\1* \2 = reinterpret_cast<\1*>(::rpgemu::DynSmem());", src)
    out, i = [], 0
    while True:
        j = src.find("<<<", i)
        if j < 0:
            out.append(src[i:])
            break
        k = _kernel_name_start(src, j)
        name = src[k:j].strip()
        e = src.index(">>>", j)
        cfg = _split_top(src[j + 3:e])
        if not 2 <= len(cfg) <= 4:
            raise ValueError(f"launch configuration of {name!r}: {cfg}")
        cfg += ["0", "nullptr"][len(cfg) - 2:]
        p = e + 3
        while src[p].isspace():
            p += 1
        if src[p] != "(":
            raise ValueError(f"no argument list after the launch of {name!r}")
        q = _match_forward(src, p, "(", ")")
        args = src[p + 1:q].strip()
        call = (f"::rpgemu::Launch(dim3({cfg[0]}), dim3({cfg[1]}), static_cast<size_t>({cfg[2]}), {cfg[3]}, "
                f"&{name}" + (f", {args}" if args else "") + ")")
        out.append(src[i:k])
        out.append(call)
        i = q + 1
    return "".join(out)


def main():
    src_path, dst_path = sys.argv[1], sys.argv[2]
    with open(src_path, encoding="utf-8-sig") as f:
        src = f.read()
    with open(dst_path, "w", encoding="utf-8") as f:
        f.write(f'#line 1 "{src_path}"\n')
        f.write(rewrite(src))


if __name__ == "__main__":
    main()
