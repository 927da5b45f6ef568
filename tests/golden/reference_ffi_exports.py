"""Writes tests/golden/reference_ffi_exports.txt: the C symbols the
reference's own library exports (every `#[no_mangle] pub ... extern "C" fn`
of its ffi/src/lib.rs), one a line. The CPU ABI test checks that
libtrit_cuda.so defines none of them.

Usage: python tests/golden/reference_ffi_exports.py <reference checkout>
"""
import os
import re
import sys


def exports(lib_rs: str) -> list[str]:
    text = open(lib_rs).read()
    names = re.findall(r"#\[no_mangle\]\s*(?:#\[[^\]]*\]\s*)*pub\s+(?:unsafe\s+)?extern\s+\"C\"\s+fn\s+(\w+)", text)
    return sorted(set(names))


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else "."
    names = exports(os.path.join(ref, "ffi", "src", "lib.rs"))
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_ffi_exports.txt")
    with open(out, "w") as f:
        f.write("\n".join(names) + "\n")
    print(f"{len(names)} names -> {out}")


if __name__ == "__main__":
    main()
