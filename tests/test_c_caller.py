"""The C ABI from a plain C11 and a C++17 caller: ``include/kvx.h`` compiles
on its own, ``_kvx.so`` links, and the entry points that need no GPU answer
as the header documents (a caller binding the library from another language
sees the same symbols)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "lmpool_b200" / "_kvx.so"

PROGRAM = r"""
#include <stdio.h>
#include "kvx.h"

int main(void) {
    int64_t ids[3] = {0, 5, 5};
    uint64_t bytes = 0;
    kvx_tuning t;
    if (kvx_abi_version() != KVX_ABI_VERSION) return 10;
    if (kvx_validate_block_ids(ids, 2, 6, 1) != KVX_OK) return 11;
    if (kvx_validate_block_ids(ids, 3, 6, 1) != KVX_EINVAL) return 12;   /* duplicate target */
    if (kvx_validate_block_ids(ids, 3, 5, 0) != KVX_EINVAL) return 13;   /* id 5 outside 5 blocks */
    if (kvx_mailbox_bytes(8, 1024, &bytes) != KVX_OK || bytes == 0) return 14;
    if (kvx_get_tuning(&t) != KVX_OK) return 15;
    printf("%s|%s|%llu\n", kvx_status_name(KVX_EINVAL), kvx_last_error(), (unsigned long long)bytes);
    return 0;
}
"""


@pytest.mark.parametrize("compiler,std,suffix", [("gcc", "-std=c11", ".c"), ("g++", "-std=c++17", ".cpp")])
def test_plain_c_and_cpp_callers_build_link_and_run(kvx_lib, tmp_path, compiler, std, suffix):
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not installed")
    src = tmp_path / f"caller{suffix}"
    src.write_text(PROGRAM)
    exe = tmp_path / "caller"
    subprocess.run([compiler, std, "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), str(LIB),
                    f"-Wl,-rpath,{LIB.parent}", "-o", str(exe)], check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    name, err, nbytes = out.stdout.strip().split("|")
    assert name and "outside" in err and int(nbytes) > 0
