"""CPU: the C-ABI library loads and exports every declared symbol.

No compute call is made here; only argument checks that return before any
device work, and the device-count query."""
import ctypes as C

import tbabi


def test_library_exports_every_header_symbol(tblib):
    lib = tblib.lib()
    names = tblib.header_symbols()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version(tblib):
    assert tblib.lib().tb_abi_version() == 1


def test_struct_layout_matches_header(tblib):
    # tb_prune_args: 8-byte aligned fields; its size is part of the ABI.
    assert C.sizeof(tbabi.PruneArgs) == 160


def test_argument_errors_return_before_device_work(tblib):
    lib = tblib.lib()
    a = tblib.prune_args(weights=1 << 20, w_dtype=0, grads=1 << 21, g_dtype=0, S=1, N=0,
                         w_out=1 << 22, mask_out=1 << 23)
    assert tblib.score_mask_pack(a) == tblib.TB_ERR_ZERO_SIZE
    a.N = 16
    a.nm_n, a.nm_m = 4, 4
    assert tblib.score_mask_pack(a) == tblib.TB_ERR_CONFIG
    a.nm_n, a.nm_m = 2, 4
    a.N = 18
    assert tblib.score_mask_pack(a) == tblib.TB_ERR_SHAPE
    a.N, a.nm_n, a.nm_m = 32, 2, 16
    assert tblib.score_mask_pack(a) == tblib.TB_ERR_UNSUPPORTED
    assert lib.tb_prepare_nm(3, 2) == tblib.TB_ERR_CONFIG
    assert b"N:M" in lib.tb_last_error()


def test_device_count_query(tblib):
    c = C.c_int(-1)
    assert tblib.lib().tb_device_count(C.byref(c)) == 0
    assert c.value >= 0
