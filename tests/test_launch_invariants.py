"""Source invariants of the launch path, checked on the CPU.

Every kernel of the library is launched with programmatic stream serialization, and
each one lets the next launch begin early (griddepcontrol.launch_dependents right
after its own wait). That is safe only while every kernel waits for its predecessor
(grid_dependency_wait) before it loads or stores memory; before the wait a kernel may
only compute addresses and ask L2 for lines (prefetch_l2). These tests read the CUDA
sources and check exactly that, and that no kernel is launched with <<<...>>>, which
would bypass the launch helper."""
import os
import re

import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baremetalinferenceengine_b200",
                    "csrc")
SOURCES = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))

# memory accesses that must not come before the wait
FORBIDDEN_BEFORE_WAIT = [
    r"\bld_stream\(", r"\bld_keep\(", r"__ldg\(", r"__ldcs\(", r"\bload1<", r"\.load\(", r"\bst_plain\(",
    r"\bst_stream\(", r"\bstore1<", r"\batomic\w*\(", r"\braise_status\(", r"\btma_\w*\(", r"\btmem_\w*\(",
    r"\bmbar\w*\(", r"\bcp\.async", r"\ba\.(positions|seq_ids|ids|lens|status)\s*\[", r"\*\s*reinterpret_cast",
]


def kernel_bodies(text):
    """(name, body) of every __global__ function definition in `text`."""
    out = []
    for m in re.finditer(r"__global__\s+void\s+(?:__\w+__\([^)]*\)\s*)*(\w+)\s*\(", text):
        i = text.find("{", m.end())
        semi = text.find(";", m.end())
        if i < 0 or (0 <= semi < i):
            continue  # a declaration, not a definition
        depth, j = 0, i
        while j < len(text):
            if text[j] == "{":
                depth += 1
            elif text[j] == "}":
                depth -= 1
                if depth == 0:
                    break
            j += 1
        out.append((m.group(1), text[i + 1:j]))
    return out


def strip_comments(text):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


ALL_KERNELS = [(os.path.basename(path), name, body) for path in SOURCES
               for name, body in kernel_bodies(strip_comments(open(path).read()))]


def test_the_sources_define_kernels():
    assert len(ALL_KERNELS) >= 20


@pytest.mark.parametrize("src,name,body", ALL_KERNELS, ids=[f"{s}:{n}" for s, n, _ in ALL_KERNELS])
def test_every_kernel_waits_before_touching_memory(src, name, body):
    k = body.find("grid_dependency_wait()")
    assert k >= 0, f"{src}: {name} never calls grid_dependency_wait()"
    before = body[:k]
    for pat in FORBIDDEN_BEFORE_WAIT:
        assert not re.search(pat, before), f"{src}: {name} matches {pat!r} before grid_dependency_wait()"


def test_no_kernel_is_launched_outside_the_launch_helper():
    for path in SOURCES:
        text = strip_comments(open(path).read())
        assert "<<<" not in text, f"{os.path.basename(path)} launches a kernel with <<<...>>>"
