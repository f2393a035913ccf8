"""CPU: the C-ABI library loads, exports every entry include/hffn_b200.h declares, and refuses bad arguments before any
launch (no GPU needed: argument checks come before the first CUDA call)."""
import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "hffn_b200.h"


def declared_entries():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z0-9_]+\s*\*?\s*(hffn_[a-z0-9_]+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_entry():
    from hffn_b200 import _native
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    names = declared_entries()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native.SIGNATURES), "ctypes signatures and header differ"


def test_version_and_policy():
    from hffn_b200 import _native as n
    assert b"sm_100a" in n.lib.hffn_version()
    assert n.lib.hffn_up_mode(1, 1024) == n.UP_CODES["coop"]
    assert n.lib.hffn_up_mode(8, 1024) == n.UP_CODES["coop"]
    assert n.lib.hffn_up_mode(9, 1024) == n.UP_CODES["tile"]
    assert n.lib.hffn_down_mode(4096, 4096) == n.DOWN_CODES["blocked"]


def test_argument_errors_before_launch():
    from hffn_b200 import _native as n
    lib = n.lib
    assert lib.hffn_forward(n.F32, None, None, None, None, None, 8, -1, -1, None) == n.HFFN_ERR_ARGUMENT
    assert b"null layer" in lib.hffn_last_error()
    layer = n.Layer(1024, 4096, 10, 10, *([1] * 8))
    assert lib.hffn_forward(7, layer, 1, 1, 1, None, 8, -1, -1, None) == n.HFFN_ERR_ARGUMENT
    assert lib.hffn_forward(n.F32, layer, 1, 1, 1, None, 0, -1, -1, None) == n.HFFN_ERR_ARGUMENT
    assert lib.hffn_up(n.F32, 9, 1, 1, 1, 1, 1, 1, None, 1024, 4096, 8, None) == n.HFFN_ERR_ARGUMENT
    assert b"up mode" in lib.hffn_last_error()
    assert lib.hffn_up(n.BF16, 0, 1, 1, 1, 1, 1, 1, 1, 1024, 4096, 8, None) == n.HFFN_ERR_ARGUMENT
    assert lib.hffn_down(n.F32, 0, 1, 1, 1, 1, 1, 1, 40000, 4096, 8, None) == n.HFFN_ERR_ARGUMENT
    assert lib.hffn_adamw(None, None, None) == n.HFFN_ERR_ARGUMENT
    assert lib.hffn_mse(None, None, None, None, 1, 1, None, None) == n.HFFN_ERR_ARGUMENT
    assert lib.hffn_backward_workspace(None, 4) == -1
    ws = lib.hffn_backward_workspace(layer, 4096)
    assert ws >= 2 * 1024 * 4096


def test_native_errors_map_to_python_exceptions():
    from hffn_b200 import _native as n
    with pytest.raises(ValueError):
        n.check(n.HFFN_ERR_ARGUMENT, "x")
    with pytest.raises(n.NativeError):
        n.check(n.HFFN_ERR_CUDA, "x")


def test_tuning_knobs_check_their_arguments():
    from hffn_b200 import _native as n
    assert n.lib.hffn_set_tc_tile_tokens(96) == n.HFFN_ERR_ARGUMENT
    assert b"tile tokens" in n.lib.hffn_last_error()
    assert n.lib.hffn_set_tc_max_ctas(-1) == n.HFFN_ERR_ARGUMENT
    for tokens in (64, 128, 256, 0):
        assert n.lib.hffn_set_tc_tile_tokens(tokens) == n.HFFN_OK
    assert n.lib.hffn_set_tc_max_ctas(0) == n.HFFN_OK


def test_peer_config_layout_matches_the_header(tmp_path):
    """The ctypes mirror of hffn_peer_config has the C layout (size and field offsets, from a probe built with gcc)."""
    import shutil
    import subprocess
    from pathlib import Path

    from hffn_b200 import _native as n
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    include = Path(n.__file__).resolve().parents[1] / "include"
    fields = ["gather", "gather_peer", "slots", "slot_peer", "partial", "signal", "signal_peer", "work"]
    probe = tmp_path / "probe.c"
    probe.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"hffn_b200.h\"\nint main(void){printf(\"%zu"
                     + " %zu" * len(fields) + "\\n\", sizeof(hffn_peer_config)"
                     + "".join(f", offsetof(hffn_peer_config, {f})" for f in fields) + ");return 0;}\n")
    subprocess.run(["gcc", f"-I{include}", str(probe), "-o", str(tmp_path / "probe")], check=True)
    c_side = [int(v) for v in subprocess.run([str(tmp_path / "probe")], capture_output=True, text=True,
                                             check=True).stdout.split()]
    py_side = [ctypes.sizeof(n.PeerConfig)] + [getattr(n.PeerConfig, f).offset for f in fields]
    assert c_side == py_side


def test_peer_entries_check_their_arguments():
    from hffn_b200 import _native as n
    handle = ctypes.c_void_p()
    cfg = n.PeerConfig()
    cfg.world, cfg.rank, cfg.tokens, cfg.dtype = 2, 2, 16, n.F32          # rank outside the world
    assert n.lib.hffn_peer_pipeline_create(ctypes.byref(cfg), ctypes.byref(n.Layer()), ctypes.byref(n.Dense()), 1,
                                           ctypes.byref(handle)) == n.HFFN_ERR_ARGUMENT
    assert n.lib.hffn_peer_pipeline_run(None, None, None, 0, None) == n.HFFN_ERR_ARGUMENT
    peers = (ctypes.c_uint64 * 2)(0, 0)
    assert n.lib.hffn_peer_barrier(1, peers, 2, 0, 1, 1000, 1, None) == n.HFFN_ERR_ARGUMENT    # rank 1's pad missing
    assert n.lib.hffn_peer_barrier(1, peers, 2, 0, 1, 0, 1, None) == n.HFFN_ERR_ARGUMENT       # no time limit
