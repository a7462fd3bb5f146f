"""The C ABI without a GPU: the library loads, exports every function that
include/sparse_decode.h declares (and the Python binding binds exactly
those), its structs have the header's layout, and argument validation
answers before any CUDA call is made."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import sparse_decode as sdp

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "sparse_decode.h"


def _header_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"#define[^\n]*", "", text)
    return set(re.findall(r"\b(sd_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def native():
    if not sdp.LIB_PATH.exists():
        from sparse_decode import build as b
        b.build()
    return sdp.lib()


def test_header_declares_what_the_binding_binds():
    assert _header_functions() == set(sdp.EXPORTED)


def test_library_exports_every_declared_function(native):
    for name in sorted(_header_functions()):
        fn = getattr(native, name)  # AttributeError when the symbol is missing
        assert ctypes.cast(fn, ctypes.c_void_p).value


def test_status_strings_and_version(native):
    assert native.sd_abi_version() >= 1
    for code, name in sdp.STATUS.items():
        s = native.sd_status_string(code).decode()
        assert s, name
    assert native.sd_status_string(99).decode()


def _c_layout(struct: str, fields: list[str]) -> dict:
    """sizeof / offsetof of a header struct, as gcc lays it out."""
    import tempfile
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields)
    src = f"""#include <stddef.h>
#include <stdio.h>
#include "sparse_decode.h"
int main(void) {{
  printf("sizeof %zu\\n", sizeof({struct}));
{body}
  return 0;
}}
"""
    with tempfile.TemporaryDirectory() as d:
        c, exe = Path(d) / "l.c", Path(d) / "l"
        c.write_text(src)
        subprocess.run(["gcc", "-std=c11", f"-I{HEADER.parent}", str(c), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.parametrize("cls,cname", [(sdp.SDConfig, "sd_config"), (sdp.SDArrays, "sd_arrays")])
def test_struct_layout_matches_header(cls, cname):
    names = [f[0] for f in cls._fields_]
    lay = _c_layout(cname, names)
    assert lay["sizeof"] == ctypes.sizeof(cls)
    for n in names:
        assert lay[n] == getattr(cls, n).offset, n


def _cfg(**kw) -> sdp.SDConfig:
    c = sdp.SDConfig()
    base = dict(batch=1, n_q_heads=32, n_kv_heads=8, head_dim=128, block_size=64, top_k=64, capacity=4096,
                dtype=2, kv_bits=0, group_size=0, shard_rank=0, shard_count=1, cluster_size=0)
    base.update(kw)
    for k, v in base.items():
        setattr(c, k, v)
    return c


BAD_CONFIGS = [
    (dict(batch=0), "SD_ERR_INVALID_ARG"),
    (dict(n_q_heads=12, n_kv_heads=8), "SD_ERR_SHAPE"),
    (dict(n_q_heads=48, n_kv_heads=3), "SD_ERR_SHAPE"),    # 16 heads per group
    (dict(head_dim=96), "SD_ERR_SHAPE"),
    (dict(block_size=48), "SD_ERR_SHAPE"),
    (dict(top_k=-1), "SD_ERR_SHAPE"),
    (dict(top_k=1024), "SD_ERR_SHAPE"),
    (dict(dtype=7), "SD_ERR_INVALID_ARG"),
    (dict(kv_bits=2), "SD_ERR_SHAPE"),
    (dict(kv_bits=4, group_size=32), "SD_ERR_SHAPE"),
    (dict(shard_count=0), "SD_ERR_INVALID_ARG"),
    (dict(shard_rank=2, shard_count=2), "SD_ERR_INVALID_ARG"),
    (dict(cluster_size=17), "SD_ERR_INVALID_ARG"),
    (dict(shard_count=16, top_k=1000), "SD_ERR_SHAPE"),   # candidate union too large
]


@pytest.mark.parametrize("kw,status", BAD_CONFIGS)
def test_create_rejects_bad_config_before_cuda(native, kw, status):
    h = ctypes.c_void_p(1)
    rc = native.sd_index_create(ctypes.byref(_cfg(**kw)), ctypes.byref(h))
    assert sdp.STATUS[rc] == status, native.sd_last_error().decode()
    assert h.value is None
    assert native.sd_last_error().decode()


def test_null_arguments(native):
    inv = "SD_ERR_INVALID_ARG"
    h = ctypes.c_void_p()
    assert sdp.STATUS[native.sd_index_create(None, ctypes.byref(h))] == inv
    assert sdp.STATUS[native.sd_index_create(ctypes.byref(_cfg()), None)] == inv
    assert native.sd_index_destroy(None) == 0
    assert sdp.STATUS[native.sd_decode(None, None, None, None, 1.0, None, None, None, None)] == inv
    assert sdp.STATUS[native.sd_append(None, None, None, 1, None)] == inv
    assert sdp.STATUS[native.sd_shard_merge(None, None, None, None, None)] == inv
    assert sdp.STATUS[native.sd_index_config(None, None)] == inv
    assert sdp.STATUS[native.sd_trim(None, 1, None)] == inv
    assert sdp.STATUS[native.sd_set_launch_overlap(None, 1)] == inv


def test_noalloc_validates_before_cuda(native):
    arr = sdp.SDArrays()
    q = ctypes.c_void_p(256)

    flags = ctypes.c_void_p(512)

    def call(cfg, off, scale=0.1, fl=flags, qq=q):
        return sdp.STATUS[native.sd_decode_noalloc(None if cfg is None else ctypes.byref(cfg), ctypes.byref(arr),
                                                   off, qq, scale, q, None, fl, None)]

    assert call(None, 1) == "SD_ERR_INVALID_ARG"
    assert call(_cfg(), 1) == "SD_ERR_INVALID_ARG"                           # k_data NULL
    assert call(_cfg(shard_count=2), 1) == "SD_ERR_STATE"                    # single-shard only
    arr.k_data = arr.v_data = arr.summaries = 256
    arr.cap_local, arr.nb_local = 4096, 64
    assert call(_cfg(kv_bits=8, group_size=64), 100) == "SD_ERR_INVALID_ARG"  # no scales / biases
    assert call(_cfg(), 0) == "SD_ERR_SHAPE"
    assert call(_cfg(), 5000) == "SD_ERR_SHAPE"
    assert call(_cfg(), 100, float("nan")) == "SD_ERR_INVALID_ARG"
    arr.nb_local = 1
    assert call(_cfg(), 100) == "SD_ERR_SHAPE"
    arr.nb_local, arr.row_bytes = 64, 128
    assert call(_cfg(), 100) == "SD_ERR_SHAPE"                               # bf16 rows are 256 B
    arr.row_bytes = 0
    assert call(_cfg(), 100, fl=None) == "SD_ERR_INVALID_ARG"                # device_flags is required
    # misaligned caller arrays are rejected on the host, before any launch
    arr.summaries = 256 + 2
    assert call(_cfg(), 100) == "SD_ERR_INVALID_ARG"
    arr.summaries, arr.k_data = 256, 256 + 8
    assert call(_cfg(), 100) == "SD_ERR_INVALID_ARG"
    arr.k_data = 256
    arr.k_scales = arr.k_biases = arr.v_scales = 1024
    arr.v_biases = 1024 + 2
    assert call(_cfg(kv_bits=8, group_size=64), 100) == "SD_ERR_INVALID_ARG"
    assert call(_cfg(), 100, qq=ctypes.c_void_p(258)) == "SD_ERR_INVALID_ARG"
