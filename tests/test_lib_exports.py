"""CPU-only checks of the C-ABI library: it loads, exports every symbol that
include/sa_b200.h declares, and its host-side validation answers without a
GPU (no compute call is made)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _header_symbols():
    text = (ROOT / "include" / "sa_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+[\s\*]+(sa_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    from smallaios_b200 import _lib

    assert _header_symbols() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    from smallaios_b200 import _lib

    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in _header_symbols() if not hasattr(raw, s)]
    assert not missing, f"missing exports: {missing}"


def test_version_and_status_strings():
    from smallaios_b200._lib import lib

    assert lib.sa_version() == 1
    assert lib.sa_status_string(0) == b"SA_OK"
    assert lib.sa_status_string(4) == b"SA_ERR_CAPACITY"


def _cfg(**kw):
    from smallaios_b200 import _lib

    c = _lib.KvCacheConfig()
    base = dict(num_layers=1, batch=1, num_heads=8, num_kv_heads=2, kv_head_begin=0, kv_head_count=2,
                head_dim=64, max_seq_len=16, bits=4, seed=42)
    base.update(kw)
    for k, v in base.items():
        setattr(c, k, v)
    return c


@pytest.mark.parametrize("kw,status,msg", [
    (dict(head_dim=48), 1, b"dim must be a power of two"),
    (dict(bits=5), 1, b"bits must be 3, 4, or 8"),
    (dict(num_layers=0), 9, b"kv_cache_allocate:zero_dim"),
    (dict(num_heads=7), 1, b"num_heads must be a positive multiple of num_kv_heads"),
    (dict(kv_head_begin=1, kv_head_count=2), 1, b"kv head range"),
    (dict(head_dim=512), 3, b"head_dim 512 outside 16..256"),
    (dict(head_dim=16, bits=3), 3, b"not a multiple of 4"),
])
def test_cache_config_validation_without_gpu(kw, status, msg):
    from smallaios_b200._lib import lib

    h = ctypes.c_void_p()
    rc = lib.sa_kv_cache_create(ctypes.byref(_cfg(**kw)), ctypes.byref(h))
    assert rc == status
    assert msg in lib.sa_last_error_string()
    assert not h.value


def test_null_handles_are_rejected():
    from smallaios_b200._lib import lib

    assert lib.sa_kv_cache_destroy(None) == 0
    assert lib.sa_kv_cache_reset(None) == 9
    assert lib.sa_group_query_attention(None, 0, None, None, None, None, 1, 1, 1, 8, 2, 0, 0.0, -1, 0, 0, None,
                                        None, 0, None) == 9


def test_matmul_nbits_validation_without_gpu():
    from smallaios_b200._lib import lib

    assert lib.sa_matmul_nbits(None, None, None, None, None, None, 1, 1, 8, 64, 3, 32, None) == 3
    assert lib.sa_matmul_nbits(None, None, None, None, None, None, 1, 1, 8, 64, 4, 24, None) == 1
    assert lib.sa_matmul_nbits(None, None, None, None, None, None, 1, 0, 8, 64, 4, 32, None) == 0
    assert lib.sa_matmul_nbits(None, None, None, None, None, None, 1, 1, 8, 64, 4, 32, None) == 9


def test_silu_mul_validation_without_gpu():
    """Shape checks of sa_silu_mul run before any launch: any row count is accepted (the kernels loop
    over rows beyond one launch's grid.y), a row shorter than its stride's half is not."""
    from smallaios_b200._lib import lib

    assert lib.sa_silu_mul(None, None, 8, None, 1, 0, 8, None) == 0          # no rows: nothing to do
    assert lib.sa_silu_mul(None, None, 4, None, 1, 70001, 8, None) == 2       # ld_in < cols
    assert lib.sa_silu_mul(None, None, 16, None, 1, 70001, 8, None) == 9      # shape fine, NULL pointers


def test_prefill_layer_rows_must_match_batch_and_prompt():
    import torch

    import smallaios_b200 as sa

    with pytest.raises(ValueError):
        sa.prefill_layer_step(torch.zeros(5, 8), None, None, None, 0, batch=2, seq_len=3)


def test_rotary_embedding_validation_without_gpu():
    from smallaios_b200 import ops
    from smallaios_b200._lib import lib

    def call(dtype=1, layout=0, heads=2, seq=4, d=64, table_dtype=1, rows=8, cols=32, pos=None, pos_dtype=7,
             pos_count=0, start=0, rdim=0, x=None):
        return lib.sa_rotary_embedding(x, x, dtype, layout, 1, heads, seq, d, None, None, table_dtype, rows, cols,
                                       pos, pos_dtype, pos_count, start, 0, rdim, None, None)

    assert call(dtype=7) == 3
    assert call(table_dtype=10) == 3
    assert call(layout=2) == 2
    assert call(heads=0) == 1
    assert call(d=63) == 2
    assert call(rdim=70) == 1 and b"rotary_dim must be in 1..=head_dim" in lib.sa_last_error_string()
    assert call(rdim=31, cols=15) == 1 and b"rotary_dim must be even" in lib.sa_last_error_string()
    assert call(cols=16) == 2 and b"cache inner dim 16" in lib.sa_last_error_string()
    assert call(start=5) == 2 and b"exceeds cos/sin table length" in lib.sa_last_error_string()
    assert call(seq=0) == 0
    assert call() == 9  # NULL tensors
    assert ops.supports_op("RotaryEmbedding")


def test_product_package_does_not_import_oracle():
    """The shipped package never reaches the CPU oracle."""
    pkg = ROOT / "smallaios_b200"
    for p in list(pkg.glob("*.py")) + list((pkg / "csrc").glob("*")):
        text = p.read_text(errors="ignore")
        assert "import oracle" not in text and "from oracle" not in text and "liboracle" not in text, p


def test_struct_layouts_match_header(tmp_path):
    """The ctypes mirrors of sa_kv_cache_config / sa_kv_layer_view have the C layout
    (sizes and field offsets from a C compiler on include/sa_b200.h)."""
    import subprocess

    from smallaios_b200 import _lib

    structs = {"sa_kv_cache_config": _lib.KvCacheConfig, "sa_kv_layer_view": _lib.KvLayerView}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "sa_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'    printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'    printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)])
    got = {}
    for line in subprocess.check_output([str(exe)], text=True).splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, f"{cname}.{f}"
