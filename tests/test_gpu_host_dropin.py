"""The reference's own backend and routed-MoE tests (tests/*.cpp of
ingeniusvictor/orbi-streammoe), compiled against the C++ drop-in layer
(orbi-streammoe_b200/host) and libosm_b200, run on the GPU with
ORBI_REQUIRE_VULKAN_COMPUTE=1 so that a missing device fails instead of
taking the tests' skip branch.  Each must print its own PASS line.  The
layer's own routed_moe_dropin_test (orbi-streammoe_b200/host/tests) checks
the drop-in's routed-MoE entry points against the reference's CPU path."""
import os
import subprocess

import pytest

from test_host_dropin import BIN, OWN_TESTS, TESTS

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", TESTS + OWN_TESTS)
def test_reference_test_passes_on_the_dropin(name):
    path = os.path.join(BIN, name)
    assert os.access(path, os.X_OK), f"{name} was not built (make -C orbi-streammoe_b200/host)"
    env = dict(os.environ, ORBI_REQUIRE_VULKAN_COMPUTE="1")
    r = subprocess.run([path], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, (name, r.stdout[-2000:], r.stderr[-2000:])
    assert ": PASS" in r.stdout and "no compute device" not in r.stdout, r.stdout
