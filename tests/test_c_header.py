"""The header is a plain C interface for C and C++ callers, not only for ctypes. A strict C11
program that includes include/sardyne_b200.h compiles without warnings. The same source compiles as
C++17. Either program links every function the header declares from the built library and runs the
host-side entry points: the version, row sizes, the GGUF reader on a file written by the package's
writer and on a missing file, and the model loader's refusals of a missing and of a malformed file
(the reference's messages, csrc/gguf.c and csrc/model_llama.c:225-319). No GPU is needed.
"""
import os
import pathlib
import shutil
import subprocess

import numpy as np
import pytest

from sardyne_b200 import capi
from sardyne_b200.gguf_writer import GGUFWriter

from test_abi import HEADER, declared_functions

pytestmark = pytest.mark.skipif(not (capi.available() and shutil.which("gcc") and shutil.which("g++")),
                                reason="needs the built library and gcc/g++")

PROGRAM = r"""
#include "sardyne_b200.h"

#include <stdio.h>
#include <string.h>

typedef void (*any_fn)(void);
static const any_fn every_function[] = {
%(functions)s
};

int main(int argc, char **argv) {
    char err[512] = "";
    size_t linked = 0;
    size_t i;
    gguf_file *g;
    int64_t k, t;
    uint64_t len = 0, blocks = 0;
    const char *arch;
    const gguf_tensor *tensor;
    engine_model *m;
    if (argc < 4) return 2;
    for (i = 0; i < sizeof every_function / sizeof every_function[0]; i++) linked += every_function[i] != NULL;
    printf("linked %%zu\n", linked);
    printf("version %%s\n", engine_version());
    printf("row_size %%zu %%zu %%zu %%zu %%zu\n", op_row_size(12, 256), op_row_size(14, 256), op_row_size(8, 32),
           op_row_size(2, 32), op_row_size(6, 32));
    g = gguf_open(argv[1], err, sizeof err);
    if (!g) {
        printf("open failed: %%s\n", err);
        return 1;
    }
    k = gguf_find_kv(g, "general.architecture");
    arch = gguf_kv_get_str(g, k, &len);
    if (gguf_kv_get_u64(g, gguf_find_kv(g, "llama.block_count"), &blocks) != 0) blocks = 0;
    t = gguf_find_tensor(g, "token_embd.weight");
    tensor = t >= 0 ? gguf_get_tensor(g, (uint64_t)t) : NULL;
    printf("gguf v%%u kv %%llu tensors %%llu arch %%.*s blocks %%llu missing_key %%lld\n", (unsigned)gguf_version(g),
           (unsigned long long)gguf_n_kv(g), (unsigned long long)gguf_n_tensors(g), (int)len, arch,
           (unsigned long long)blocks, (long long)gguf_find_kv(g, "no.such.key"));
    if (tensor)
        printf("tensor %%s %%s %%llux%%llu bytes %%llu\n", tensor->name, gguf_type_name(tensor->type),
               (unsigned long long)tensor->ne[0], (unsigned long long)tensor->ne[1],
               (unsigned long long)tensor->nbytes);
    gguf_close(g);
    err[0] = 0;
    g = gguf_open(argv[2], err, sizeof err);
    printf("missing gguf %%s: %%s\n", g ? "opened" : "refused", err);
    err[0] = 0;
    m = engine_model_load(argv[2], err, sizeof err);
    printf("missing model %%s: %%s\n", m ? "loaded" : "refused", err);
    err[0] = 0;
    m = engine_model_load(argv[3], err, sizeof err);
    printf("bad model %%s: %%s\n", m ? "loaded" : "refused", err);
    sdy_clear_error();
    printf("error after clear: [%%s]\n", sdy_last_error());
    return 0;
}
"""


def build_and_run(tmp_path, compiler, std, suffix):
    src = tmp_path / f"caller.{suffix}"
    src.write_text(PROGRAM % {"functions": "\n".join(f"    (any_fn){n}," for n in declared_functions())})
    exe = tmp_path / f"caller_{suffix}"
    lib_dir = pathlib.Path(capi.lib_path()).parent
    cmd = [compiler, f"-std={std}", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(HEADER.parent), str(src),
           "-o", str(exe), "-L", str(lib_dir), "-lsardyne", f"-Wl,-rpath,{lib_dir}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-4000:]
    good = GGUFWriter(tmp_path / "good.gguf")
    good.add("general.architecture", "llama")
    good.add("llama.block_count", 3)
    good.add_tensor("token_embd.weight", np.zeros((8, 32), np.float32))
    bad = GGUFWriter(tmp_path / "bad.gguf")
    bad.add("general.architecture", "qwen3moe")
    for key, value in [("embedding_length", 32), ("block_count", 1), ("feed_forward_length", 64),
                       ("attention.head_count", 2), ("expert_count", 4), ("expert_used_count", 5)]:
        bad.add(f"qwen3moe.{key}", value)
    bad.add_tensor("token_embd.weight", np.zeros((8, 32), np.float32))
    env = dict(os.environ, LD_LIBRARY_PATH=str(lib_dir))
    r = subprocess.run([str(exe), str(good.write()), str(tmp_path / "missing.gguf"), str(bad.write())],
                       capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout.splitlines()


@pytest.mark.parametrize("compiler,std,suffix", [("gcc", "c11", "c"), ("g++", "c++17", "cpp")])
def test_c_caller_compiles_links_and_runs(tmp_path, compiler, std, suffix):
    out = build_and_run(tmp_path, compiler, std, suffix)
    assert out[0] == f"linked {len(declared_functions())}"
    assert out[1] == "version 0.0.1"
    assert out[2] == "row_size 144 210 34 18 22"  # Q4_K, Q6_K, Q8_0, Q4_0, Q5_0 rows of one block
    assert out[3] == "gguf v3 kv 2 tensors 1 arch llama blocks 3 missing_key -1"
    assert out[4] == "tensor token_embd.weight F32 32x8 bytes 1024"
    assert out[5].startswith("missing gguf refused: ") and "impossibile aprire" in out[5]
    assert out[6].startswith("missing model refused: ") and "impossibile aprire" in out[6]
    assert out[7].startswith("bad model refused: ") and "expert_used_count=5 oltre expert_count=4" in out[7]
    assert out[8] == "error after clear: []"
