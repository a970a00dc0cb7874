"""The C-ABI library loads, exports every entry point include/q3attn.h
declares, and its q3a_cfg layout matches the header.  No compute call: these
run on a CPU-only machine too."""
import ctypes
import os
import re
import subprocess

import pytest

import q3attn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "q3attn.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(q3a_[a-z_0-9]+)\s*\(", src)))


def test_header_lists_the_binding_exports():
    assert header_functions() == sorted(q3attn.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = q3attn.load()
    for name in header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", q3attn.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (q3a_\w+)", out))
    assert set(header_functions()) <= exported


def test_cfg_layout_matches_header():
    """Compiles a probe against the header and compares sizeof/offsets."""
    import tempfile
    probe = r'''
#include <stdio.h>
#include <stddef.h>
#include "q3attn.h"
int main(void){
  printf("%zu %zu %zu %zu\n", sizeof(q3a_cfg), offsetof(q3a_cfg, norm_eps),
         offsetof(q3a_cfg, kv_head_begin), offsetof(q3a_cfg, kv_head_count));
  return 0; }
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "p.c")
        exe = os.path.join(d, "p")
        open(c, "w").write(probe)
        subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), c, "-o", exe],
                       check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                               check=True).stdout.split()]
    C = q3attn.Cfg
    assert vals == [ctypes.sizeof(C), C.norm_eps.offset, C.kv_head_begin.offset,
                    C.kv_head_count.offset]


def test_cfg_defaults_are_qwen3_8b():
    c = q3attn.default_cfg()
    assert (c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim) == (36, 32, 8, 128)
    assert c.rope_theta == pytest.approx(5e6) and c.norm_eps == pytest.approx(1e-6)


def test_create_rejects_bad_shapes_without_gpu_work():
    """Shape validation happens before any device call, so it runs anywhere."""
    lib = q3attn.load()
    for kw in ({"head_dim": 64}, {"n_heads": 16}, {"page_tokens": 48}):
        cfg = q3attn.default_cfg(**kw)
        h = ctypes.c_void_p()
        rc = lib.q3a_create(ctypes.byref(h), ctypes.byref(cfg))
        assert rc in (q3attn.ERR_UNSUPPORTED, q3attn.ERR_INVALID)
        assert lib.q3a_last_error().decode() != ""


def test_c_host_links_and_calls_the_library(tmp_path):
    """A C host, as the reference's main.c would be: includes the header,
    links libq3attn.so, fills the default configuration and gets a clean
    error for an unsupported shape (no device work)."""
    lib_dir = os.path.dirname(q3attn.LIB_PATH)
    src = tmp_path / "host.c"
    src.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "q3attn.h"
int main(void) {
    q3a_cfg cfg;
    q3a_cfg_default(&cfg);
    if (cfg.n_heads != 32 || cfg.n_kv_heads != 8 || cfg.head_dim != 128) return 2;
    cfg.head_dim = 64;
    q3a_ctx *ctx = NULL;
    int rc = q3a_create(&ctx, &cfg);
    if (rc != Q3A_ERR_UNSUPPORTED || ctx != NULL || strlen(q3a_last_error()) == 0) return 3;
    printf("ok %s\n", q3a_last_error());
    return 0;
}
""")
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                    "-L", lib_dir, "-lq3attn", "-Wl,-rpath," + lib_dir], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok ")
