"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, validates before launching (the reference rejects bad
dispatch shapes before allocation, metal.rs:945-956), and implements the
decision rule of answers() (crates/core/src/types.rs:728-802)."""
import ctypes
import math
import re
from pathlib import Path

import numpy as np
import pytest

import clef_b200 as cb
from clef_b200.config import benchmark_config

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "clef_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(clef_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    declared = header_functions()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(cb.lib, name), name
    assert sorted(cb.EXPORTS) == declared
    assert "sm_100a" in cb.version()


def test_config_validation():
    cfg = benchmark_config()
    assert cb.lib.clef_config_validate(ctypes.byref(cfg)) == 0
    bad = benchmark_config()
    bad.linear_key_head_dim = 64
    assert cb.lib.clef_config_validate(ctypes.byref(bad)) == 3
    bad = benchmark_config()
    bad.num_attention_heads = 15
    assert cb.lib.clef_config_validate(ctypes.byref(bad)) == 1
    assert cb.lib.clef_config_validate(None) == 1


FAKE = ctypes.c_void_p(0x10000)  # never dereferenced: every call below fails validation first


def test_delta_scan_rejects_before_launch():
    L = cb.lib
    args = dict(T=64, Hk=16, Hv=32, dk=128, dv=128)
    # null pointers
    assert L.clef_delta_scan(None, FAKE, FAKE, FAKE, FAKE, 64, 16, 32, 128, 128, None, 1, None, 0, 0,
                             None, None, FAKE, FAKE, 1 << 30, None) == 1
    # unsupported head dims (metal.rs dimensions(): key must be a power of two <= 128)
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 64, 16, 32, 127, 128, None, 1, None, 0, 0,
                             None, None, FAKE, FAKE, 1 << 30, None) == 3
    # head counts that do not divide
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 64, 3, 32, 128, 128, None, 1, None, 0, 0,
                             None, None, FAKE, FAKE, 1 << 30, None) == 1
    # empty sequence
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 0, 16, 32, 128, 128, None, 1, None, 0, 0,
                             None, None, FAKE, FAKE, 1 << 30, None) == 1
    # capture without a destination
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 64, 16, 32, 128, 128, None, 1, None, 0, 5,
                             None, None, FAKE, FAKE, 1 << 30, None) == 1
    # capture past the end
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 64, 16, 32, 128, 128, None, 1, None, 0, 65,
                             FAKE, None, FAKE, FAKE, 1 << 30, None) == 1
    # unordered cu_seqlens
    cu = np.array([0, 40, 30, 64], np.int64)
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 64, 16, 32, 128, 128, cu.ctypes.data, 3,
                             None, 0, 0, None, None, FAKE, FAKE, 1 << 30, None) == 1
    # workspace too small for the offsets of three sequences
    cu = np.array([0, 10, 30, 64], np.int64)
    assert L.clef_delta_scan(FAKE, FAKE, FAKE, FAKE, FAKE, 64, 16, 32, 128, 128, cu.ctypes.data, 3,
                             None, 0, 0, None, None, FAKE, ctypes.c_void_p(0x20000), 16, None) == 1
    assert "workspace" in cb.lib.clef_last_error().decode()
    assert args


def test_workspace_size():
    # Chunk tables plus, per 64-token chunk, 64 KB of split K/Q tiles per key
    # head and 34048 bytes of solved tiles and decay vectors per value head.
    a = cb.delta_scan_workspace_size(1024, 1, 16, 32)
    b = cb.delta_scan_workspace_size(2048, 1, 16, 32)
    assert 0 < a < b
    per_chunk = 16 * 65536 + 32 * 34048
    assert per_chunk * 16 <= b - a <= per_chunk * 16 + 4096
    assert cb.delta_scan_workspace_size(1024, 1, 16, 32, dk=64) == 0
    assert cb.delta_scan_workspace_size(-1, 1, 16, 32) == 0


def test_gemm_rejects_before_launch():
    L = cb.lib
    assert L.clef_gemm_bf16(FAKE, FAKE, 128, 256, 100, 0, FAKE, 256, None) == 3  # K % 64
    assert L.clef_gemm_bf16(FAKE, FAKE, 128, 250, 128, 0, FAKE, 256, None) == 3  # N % 16
    assert L.clef_gemm_bf16(FAKE, FAKE, 128, 256, 128, 7, FAKE, 256, None) == 1  # epilogue
    assert L.clef_gemm_bf16(FAKE, FAKE, 128, 256, 128, 0, FAKE, 100, None) == 1  # ldo < N
    assert L.clef_gemm_bf16(None, FAKE, 128, 256, 128, 0, FAKE, 256, None) == 1
    assert L.clef_gemm_swiglu(FAKE, FAKE, None, 128, 256, 128, FAKE, None) == 1


def test_attention_and_pointwise_reject_before_launch():
    L = cb.lib
    assert L.clef_attention_gqa(FAKE, FAKE, FAKE, 16, 4, 10, 10, 128, FAKE, FAKE, 1 << 30, None) == 3
    assert L.clef_attention_gqa(FAKE, FAKE, FAKE, 16, 5, 10, 10, 256, FAKE, FAKE, 1 << 30, None) == 1
    assert L.clef_attention_gqa(FAKE, FAKE, FAKE, 16, 4, 11, 10, 256, FAKE, FAKE, 1 << 30, None) == 1
    # A workspace smaller than clef_attention_gqa_workspace_size is refused.
    need = L.clef_attention_gqa_workspace_size(16, 4, 10, 10)
    assert need > 0
    assert L.clef_attention_gqa(FAKE, FAKE, FAKE, 16, 4, 10, 10, 256, FAKE, FAKE, need - 1, None) == 1
    assert L.clef_rmsnorm(FAKE, FAKE, 4, 256, 0.0, 0, FAKE, None) == 1
    assert L.clef_rmsnorm(FAKE, FAKE, 4, 256, 1e-6, 5, FAKE, None) == 1
    assert L.clef_conv4(FAKE, 8, None, 2, FAKE, 4, 8, FAKE, None) == 1  # history rows without data
    assert L.clef_delta_prologue(FAKE, 12352, 12288, 12320, None, 0, FAKE, FAKE, FAKE, 8, 16, 32, 64,
                                 128, FAKE, FAKE, FAKE, FAKE, FAKE, None) == 3
    assert L.clef_compact_copy(FAKE, 5, FAKE, FAKE, 4, FAKE, None) == 1


def test_engine_reports_missing_device_or_bad_config():
    cfg = benchmark_config()
    cfg.linear_conv_kernel_dim = 3
    h = ctypes.c_void_p()
    assert cb.lib.clef_engine_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == 3
    assert not h.value


def answers_reference(logits):
    """answers() restated: softmax with max subtraction, first strict max wins."""
    out = []
    for l in np.asarray(logits, np.float32).reshape(-1, 7):
        def softmax(x):
            m = np.float32(max(x))
            p = [np.float32(math.exp(np.float32(v - m))) for v in x]
            s = np.float32(sum(p))
            return [np.float32(v / s) for v in p]
        pn, pc = softmax(l[:2]), softmax(l[2:6])
        best, win = -1.0, -1
        for i, p in enumerate(pc):
            if p > best:
                best, win = p, i
        out.append((pn[0], win, best, l[6]))
    return out


def test_decide_matches_answers_rule():
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((64, 7)).astype(np.float32)
    lg[5, 2:6] = [1.0, 3.0, 3.0, 0.5]   # tie: the first maximum wins
    lg[6, 2:6] = [2.0, 2.0, 2.0, 2.0]
    got = cb.decide(lg)
    ref = answers_reference(lg)
    for d, (noul, win, conf, score) in zip(got, ref):
        assert d.choice == win
        assert abs(d.noul - noul) < 1e-6 and abs(d.confidence - conf) < 1e-6
        assert d.score == score
    assert got[5].choice == 1 and got[6].choice == 0
    bad = lg.copy()
    bad[0, 0] = np.inf
    with pytest.raises(cb.ClefError):
        cb.decide(bad)


def test_head_rejects_bad_geometry_before_touching_a_device():
    """clef_head_create validates HeadConfig (head.rs:26-47) before any CUDA
    call: head width must divide 256, dimensions positive, handle required."""
    L = cb.lib
    h = ctypes.c_void_p()
    cfg = cb.HeadConfig(hidden_size=2560, width=1024, routing_layers=2, layers=4, heads=16, feedforward=4096)
    assert L.clef_head_create(None, 0, ctypes.byref(h)) == 1
    bad = cb.HeadConfig(hidden_size=2560, width=1000, routing_layers=2, layers=4, heads=16, feedforward=4096)
    assert L.clef_head_create(ctypes.byref(bad), 0, ctypes.byref(h)) == 3
    bad = cb.HeadConfig(hidden_size=0, width=1024, routing_layers=2, layers=4, heads=16, feedforward=4096)
    assert L.clef_head_create(ctypes.byref(bad), 0, ctypes.byref(h)) == 1
    assert L.clef_head_create(ctypes.byref(cfg), 0, None) == 1
    assert L.clef_head_set_weight(None, b"x", FAKE, 1) == 1
    assert L.clef_head_finalize(None) == 1
    assert L.clef_head_destroy(None) == 0


def test_selftest_rejects_bad_limit_before_launch():
    assert cb.lib.clef_selftest_wait_timeout(0, None) == 1
    assert cb.lib.clef_selftest_wait_timeout(5000, None) == 1


def test_prefix_transfer_rejects_before_touching_a_device():
    lib = cb.lib
    buf = ctypes.create_string_buffer(16)
    assert lib.clef_prefix_span_bytes(None) == 0
    assert lib.clef_prefix_export(None, buf, 16, None) == 1
    assert "null pointer" in lib.clef_last_error().decode()
    assert lib.clef_prefix_import(None, buf, 16, None) == 1
    out = ctypes.c_void_p(0x1)
    assert lib.clef_prefix_create(None, 16, ctypes.byref(out)) == 1
    assert out.value is None  # cleared on every path


def test_delta_packed_rejects_the_reference_dimension_limits():
    """clef_delta_packed refuses what the reference's `dimensions` refuses
    (metal.rs:280-290) before touching device memory."""
    import clef_b200 as cb
    fake = ctypes.c_void_p(0x10000)
    L = cb.lib
    for T, H, dk, dv, cap in [(0, 1, 4, 4, 0), (4097, 1, 4, 4, 0), (8, 33, 4, 4, 0), (8, 2, 3, 4, 0),
                              (8, 2, 256, 4, 0), (8, 2, 4, 129, 0), (8, 2, 4, 0, 0), (8, 2, 4, 4, 9)]:
        assert L.clef_delta_packed(fake, T, H, dk, dv, None, cap, fake, None) == 1, (T, H, dk, dv, cap)
    assert "dimensions" in L.clef_last_error().decode() or "capture" in L.clef_last_error().decode()
    assert L.clef_delta_prepare_packed(fake, 8192, fake, fake, 4097, 16, 32, fake, None) == 1


def test_precision_setter_validates_before_touching_an_engine():
    import clef_b200 as cb
    assert cb.lib.clef_engine_set_precision(None, 1) == 1
    assert cb.lib.clef_engine_precision(None) == -1
    assert cb.PRECISION_BF16 == 0 and cb.PRECISION_SPLIT == 1


def test_header_is_plain_c_and_a_c_caller_links_every_entry(tmp_path):
    """The header compiles as strict C11 (what bindgen or cgo read) and a C
    program that takes the address of every declared entry links against
    libclef_b200.so and runs its host-only entries, as a foreign caller would."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    names = header_functions()
    table = ",\n".join(f'  {{"{n}", (fn)&{n}}}' for n in names)
    src = tmp_path / "caller.c"
    src.write_text(f"""#include "clef_b200.h"
#include <stdio.h>
#include <string.h>
typedef void (*fn)(void);
static const struct {{ const char* name; fn f; }} table[] = {{
{table}
}};
int main(void) {{
  size_t i;
  float logits[7] = {{0.5f, -0.5f, 1.0f, 3.0f, 3.0f, 0.5f, 2.0f}};
  clef_decision d;
  for (i = 0; i < sizeof table / sizeof table[0]; ++i)
    if (!table[i].f) return 10;
  if (!strstr(clef_version(), "sm_100a")) return 11;
  if (clef_config_validate(NULL) == 0) return 12;
  if (strlen(clef_last_error()) == 0) return 13;
  if (clef_decide(logits, 1, 7, &d) != 0) return 14;
  if (d.choice != 1) return 15; /* the first of two equal maxima */
  printf("%d entries\\n", (int)(sizeof table / sizeof table[0]));
  return 0;
}}
""")
    lib_dir = cb.LIB_PATH.parent
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I", str(ROOT / "include"), str(src), "-L", str(lib_dir), "-lclef_b200",
                    f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.strip() == f"{len(names)} entries"
