"""Rewrites HIP kernel launches `kernel<<<grid, block, smem, stream>>>(args)` of a reference
source file into `::simsim::launch(grid, block, smem, stream).run(kernel, args)`, the host
SIMT emulator's launch (oracle/hipsim/hip/hip_runtime.h) -- TEST INFRASTRUCTURE ONLY. The
output goes to oracle/_build/ and is compiled by oracle/Makefile; nothing else in the source
changes.

    python hip_to_host.py IN OUT
"""
import re
import sys

LAUNCH = re.compile(r"([A-Za-z_][\w:]*(?:<[^<>;()]*>)?)\s*<<<(.*?)>>>\s*\(")


def rewrite(text: str) -> str:
    return LAUNCH.sub(lambda m: f"::simsim::launch({m.group(2)}).run({m.group(1)}, ", text)


if __name__ == "__main__":
    src, dst = sys.argv[1], sys.argv[2]
    with open(src) as f:
        text = f.read()
    out = rewrite(text)
    if "<<<" in out:
        sys.exit(f"{src}: a launch the rewrite does not recognise remains")
    with open(dst, "w") as f:
        f.write(f"// generated from {src.rsplit('/', 1)[-1]} by oracle/hip_to_host.py: kernel launches rewritten for the host emulator\n")
        f.write(f'#line 1 "{src.rsplit("/", 1)[-1]}"\n')
        f.write(out)
