"""The C++ drop-in layer (orbi-streammoe_b200/host): the reference's backend
classes over libosm_b200's C ABI, and the reference's own backend and
routed-MoE tests compiled against it.

CPU checks: every public function and class of the reference backend headers
the model layer includes is declared, with the same parameter list, by the
drop-in headers; the test binaries were built and, without a GPU, take the
reference tests' own "no compute device" branch.  On a GPU the same binaries
run with ORBI_REQUIRE_VULKAN_COMPUTE=1 (test_gpu_host_dropin.py).
"""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "orbi-streammoe_b200", "host")
BIN = os.path.join(HOST, "_build", "bin")
REF = os.environ.get("OSM_REFERENCE_ROOT", "/root/reference")
HEADERS = sorted(os.listdir(os.path.join(HOST, "include", "orbi", "streammoe", "backend")))
_MAKEFILE = open(os.path.join(HOST, "Makefile")).read()
TESTS = re.search(r"\nTESTS := \\\n(.*?)\n\n", _MAKEFILE, re.S).group(1).replace("\\", " ").split()
# this layer's own tests (host/tests/*.cpp): the drop-in against the
# reference's CPU path
OWN_TESTS = re.search(r"\nOWN_TESTS := ([^\n]*)", _MAKEFILE).group(1).split()


def _drop_private(text):
    """Removes each private: section up to the closing brace of its class."""
    while "private:" in text:
        i = text.index("private:")
        depth, j = 0, i
        while j < len(text):
            if text[j] == "{":
                depth += 1
            elif text[j] == "}":
                if depth == 0:
                    break
                depth -= 1
            j += 1
        text = text[:i] + text[j:]
    return text


def _public_decls(text):
    """Normalised declarations of free functions and member functions."""
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"\s+", " ", text)
    text = _drop_private(text)
    out = set()
    for m in re.finditer(r"(\[\[nodiscard\]\] )?([\w:<>,\* &]+?) (\w+)\(([^()]*(?:\([^()]*\))?[^()]*)\)"
                         r"( const)?( noexcept)?[ ;=]", text):
        name, params = m.group(3), m.group(4)
        if name in ("if", "for", "while", "return", "sizeof", "static_cast", "alignas"):
            continue
        params = re.sub(r" = [^,]*", "", params)        # default arguments
        params = re.sub(r"\b(\w+)\s*(,|$)", r"\2", params)  # parameter names
        params = re.sub(r"\s+", " ", params).strip()
        out.add((name, params, bool(m.group(5))))
    return out


def _reference_available():
    return os.path.exists(os.path.join(REF, "include", "orbi", "streammoe", "backend"))


@pytest.mark.parametrize("header", HEADERS)
def test_headers_declare_the_reference_interface(header):
    if not _reference_available():
        pytest.skip("reference headers not present")
    ref = _public_decls(open(os.path.join(REF, "include/orbi/streammoe/backend", header)).read())
    ours = _public_decls(open(os.path.join(HOST, "include/orbi/streammoe/backend", header)).read())
    missing = sorted(d for d in ref if d not in ours)
    assert not missing, f"{header}: reference declarations missing from the drop-in: {missing}"


def test_dropin_binaries_built_and_skip_without_gpu():
    if not _reference_available():
        pytest.skip("reference sources not present: binaries are built in the source container")
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present: test_gpu_host_dropin.py runs the binaries")
    for t in TESTS + OWN_TESTS:
        path = os.path.join(BIN, t)
        assert os.access(path, os.X_OK), f"{t} not built (make -C orbi-streammoe_b200/host)"
        r = subprocess.run([path], capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, (t, r.stdout, r.stderr)
        assert "PASS (no compute device on host)" in r.stdout, (t, r.stdout)
        # and where the test honours it, a required device that is missing is
        # an error, not a pass
        src = os.path.join(HOST, "tests", t + ".cpp") if t in OWN_TESTS else os.path.join(REF, "tests", t + ".cpp")
        if "ORBI_REQUIRE_VULKAN_COMPUTE" not in open(src).read():
            continue
        env = dict(os.environ, ORBI_REQUIRE_VULKAN_COMPUTE="1")
        r = subprocess.run([path], capture_output=True, text=True, timeout=120, env=env)
        assert r.returncode != 0, (t, r.stdout)
