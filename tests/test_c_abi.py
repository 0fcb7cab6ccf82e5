"""The boundary from C: include/hymoe.h compiles as C99 with every warning an error
(-Wall -Wextra -pedantic -Werror), a C program links against libhymoe.so, and the entry points
that need no device (statuses on NULL, the placement helper, the GGUF reader on a file written
by gguf-py) behave as documented.  No GPU needed."""
import os
import shutil
import subprocess

import pytest

import hymoe
import oracle as O
from moe_cases import host_layer

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_consumer_compiles_links_and_runs(tmp_path):
    pytest.importorskip("gguf")
    from gguf_layer import write_moe_layer
    orc = O.Oracle()
    H, I, E = 256, 128, 8
    lay = host_layer(orc, 5, 0, H, I, E, O.Q4_0)
    path = str(tmp_path / "layer.gguf")
    write_moe_layer(path, 3, H, I, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], O.Q4_0)
    exe = str(tmp_path / "consumer")
    lib_dir = os.path.dirname(hymoe.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", os.path.dirname(hymoe.HEADER), os.path.join(HERE, "c_abi", "consumer.c"),
                    "-o", exe, "-L", lib_dir, "-l:libhymoe.so", f"-Wl,-rpath,{lib_dir}", "-lm"],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([exe, path], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
