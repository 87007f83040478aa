"""register() against a stand-in tinygrad package (tests/stub_tinygrad): the reference's
registration steps (tinygrad-dx12 src/tinygrad_dx12/compat.py:93-96,175-176) -- the device
module importable under tinygrad's name, the device appended to Device._devices and put first
in ALL_DEVICES -- happen once however often register() runs (idempotence as in the reference's
test/device/test_compat.py:47-64). Each case runs in a fresh interpreter so the real import of
tinygrad_dx12_b200 (which registers on import) sees the stand-in."""

import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent
STUB = ROOT / "tests" / "stub_tinygrad"


def _run(code: str, with_stub: bool = True) -> str:
    path = [str(STUB)] if with_stub else []
    prog = "import sys; sys.path[:0] = %r; sys.path.insert(0, %r)\n" % (path, str(ROOT)) + code
    res = subprocess.run([sys.executable, "-c", prog], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    return res.stdout.strip()


def test_register_fills_the_device_tables_once():
    out = _run(
        "import tinygrad_dx12_b200 as tg\n"
        "from tinygrad.device import Device, ALL_DEVICES\n"
        "tg.register(); tg.register()\n"
        "import tinygrad.runtime.ops_b200 as m\n"
        "print(Device._devices.count('B200'), ALL_DEVICES[0], ALL_DEVICES.count('B200'), m.B200Device.__name__,"
        " m.B200Device('B200:1').device, tg.compat.registered())\n")
    assert out == "1 B200 1 B200Device B200:1 True"


def test_register_without_tinygrad_opens_nothing():
    out = _run(
        "import importlib.util\n"
        "assert importlib.util.find_spec('tinygrad') is None\n"
        "import tinygrad_dx12_b200 as tg\n"
        "tg.register()\n"
        "import sys\n"
        "print(tg.compat.registered(), 'tinygrad.runtime.ops_b200' in sys.modules)\n", with_stub=False)
    assert out == "True False"
