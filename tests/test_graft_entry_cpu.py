"""The build entry point the driver calls: ``build()`` compiles the extension
in-tree and imports it in a fresh interpreter (where ``bwn._C`` needs
torch's shared libraries loaded first)."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_build_entry_point_imports_the_extension():
    r = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.build(); print('BUILD_OK')"],
                       cwd=ROOT, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0 and "BUILD_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]
