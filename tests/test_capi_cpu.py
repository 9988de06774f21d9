"""The C-ABI library on a machine without a GPU: it loads, exports every
symbol include/mxg.h declares, and rejects bad arguments on the host before
any CUDA call."""


def test_library_loads_and_exports_header_symbols(mxg):
    L = mxg._lib.load()
    syms = mxg._lib.header_symbols()
    assert len(syms) >= 13
    for s in syms:
        assert hasattr(L, s), f"{s} missing from libmxg.so"
    assert set(syms) == set(mxg._lib._PROTOS), "ctypes prototypes out of sync with include/mxg.h"


def test_error_strings(mxg):
    L = mxg._lib.load()
    assert L.mxg_error_string(0) == b"ok"
    assert b"offsets" in L.mxg_error_string(7)
    assert L.mxg_error_string(999) == b"unknown error"
    assert L.mxg_version() >= 100


def test_workspace_sizes(mxg):
    L = mxg._lib.load()
    fwd = L.mxg_grouped_fwd_workspace_size(32, 66560, 4096, 7168)
    # A-side scales: 32 experts x 32 row blocks x 56 K blocks x 512 B
    assert fwd >= 32 * 32 * 56 * 512
    assert fwd < 256 << 20
    wg = L.mxg_grouped_wgrad_workspace_size(32, 66560, 4096, 7168)
    assert wg > 0 and wg < 256 << 20
    assert L.mxg_grouped_fwd_workspace_size(0, 1, 1, 32) == 0


def _fwd(L, **kw):
    args = dict(a=16, a_scales=None, w=16, w_scales=None, offs=None, offs_len=0, offs_kind=3,
                E=1, m=64, n=64, k=64, out=16, dtype=0, ws=16, ws_bytes=1 << 20, stream=None)
    args.update(kw)
    return L.mxg_grouped_fwd(args["a"], args["a_scales"], args["w"], args["w_scales"], args["offs"],
                             args["offs_len"], args["offs_kind"], args["E"], args["m"], args["n"],
                             args["k"], args["out"], args["dtype"], args["ws"], args["ws_bytes"],
                             args["stream"])


def test_host_validation_without_gpu(mxg):
    L = mxg._lib.load()
    assert _fwd(L, k=48) == 2                      # K not a multiple of 32
    assert _fwd(L, E=0) == 1                       # no groups
    assert _fwd(L, E=300, offs=16, offs_len=300) == 9  # too many groups
    assert _fwd(L, E=2) == 1                       # offs required for E > 1
    assert _fwd(L, E=2, offs=16, offs_len=5, offs_kind=0) == 1  # [E+1] length mismatch
    assert _fwd(L, dtype=7) == 1                   # unknown output dtype
    assert _fwd(L, a=17) == 3                      # misaligned
    assert _fwd(L, m=0) == 0                       # empty problem: no work
    assert L.mxg_quantize_rowwise(16, 4, 48, 16, 16, None) == 2
    assert L.mxg_quantize_colwise(16, 48, 4, 16, 16, None) == 2
    assert L.mxg_quantize_rowwise(None, 4, 64, 16, 16, None) == 1
    assert L.mxg_grouped_wgrad(16, None, 16, None, 16, 2, 2, 2, 100, 64, 64, 16, 0, 16, 1 << 20, None) == 2
    assert L.mxg_debug_inject_stall(-1) == 1
    assert L.mxg_debug_inject_stall(0) == 0


def test_status_codes_match_header(mxg):
    import re
    text = open(mxg._lib.HEADER_PATH).read()
    codes = dict(re.findall(r"#define (MXG_(?:OK|ERR_\w+))\s+(\d+)", text))
    assert codes, "no status codes found in the header"
    for name, value in codes.items():
        assert getattr(mxg._lib, name) == int(value), name
