"""Source invariants behind programmatic dependent launch, checked on the CPU.

A kernel may be scheduled while the kernel before it in the stream is still running; it is correct
only if it waits on the device (qb_pdl_wait, griddepcontrol.wait) before touching memory that
earlier work writes, and before it can exit -- a kernel that finished without waiting would let the
kernel after it pass its own wait too early.  Every launch goes through qb_launch / qb_launch_ex,
which set the launch attributes in one place.  These checks read the CUDA sources.
"""
import re
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "qwen3_naive_inference_b200" / "csrc"


def _kernels(text):
    """(name, body) of every __global__ function, the body from its opening brace to the match."""
    out = []
    for m in re.finditer(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s*)?([A-Za-z_]\w*)\s*\(", text):
        i = text.index("{", m.end())
        depth, j = 0, i
        while True:
            if text[j] == "{":
                depth += 1
            elif text[j] == "}":
                depth -= 1
                if depth == 0:
                    break
            j += 1
        out.append((m.group(1), text[i + 1:j]))
    return out


def test_every_kernel_waits_before_any_return():
    n = 0
    for f in sorted(CSRC.glob("*.cu")):
        text = f.read_text()
        for name, body in _kernels(text):
            n += 1
            # lambdas' own returns (barrier-address helpers) are not the kernel's
            flat = re.sub(r"\[[^\]]*\]\s*\([^)]*\)\s*\{[^{}]*\}", "LAMBDA", body)
            w = flat.find("qb_pdl_wait()")
            assert w >= 0, f"{f.name}:{name} never calls qb_pdl_wait()"
            r = re.search(r"\breturn\b", flat)
            assert r is None or r.start() > w, f"{f.name}:{name} can return before qb_pdl_wait()"
    assert n >= 30  # every kernel of the library was seen


def test_every_launch_goes_through_the_launch_helper():
    for f in sorted(CSRC.glob("*.cu")):
        text = f.read_text()
        assert "<<<" not in text, f"{f.name}: a <<< >>> launch bypasses qb_launch"
        assert "cudaLaunchKernelEx(" not in text, f"{f.name}: cudaLaunchKernelEx outside qb_launch"


def test_tmem_kernels_trigger_only_after_their_allocation():
    """A kernel holding TMEM lets the next kernel start only once its own allocation succeeded."""
    for f in sorted(CSRC.glob("*.cu")):
        for name, body in _kernels(f.read_text()):
            a = body.find("tcgen05.alloc")
            if a < 0:
                continue
            t = body.find("qb_pdl_trigger()")
            assert t > a, f"{f.name}:{name} triggers its dependents before allocating TMEM"
