"""The C-ABI library loads and exports every function include/mserve_kv.h declares; the ctypes
layouts in mserve_b200/_lib.py match the header's structs; host-side argument errors are raised
before any GPU work.  CPU only (no kernel is launched)."""
import ctypes as C
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "mserve_kv.h"


def _declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(mskv_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_every_declared_function_is_exported(built_lib):
    lib = C.CDLL(str(built_lib))
    names = _declared_functions()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_bindings_cover_the_header(built_lib):
    from mserve_b200 import _lib
    bound = {name for name, _, _ in _lib.SIGNATURES}
    declared = set(_declared_functions())
    assert bound <= declared
    lib = _lib.lib()
    assert lib.mskv_abi_version() == 2
    assert isinstance(_lib.launch_count(), int)


def _c_struct_fields(name):
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    m = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, flags=re.S)
    assert m, name
    fields = []
    for line in m.group(1).split(";"):
        line = line.strip()
        if line:
            fields.append(line.split()[-1].lstrip("*"))
    return fields


@pytest.mark.parametrize("cname,pyname", [("mskv_rows", "Rows"), ("mskv_gather_desc", "GatherDesc"),
                                          ("mskv_copy_desc", "CopyDesc"), ("mskv_score_desc", "ScoreDesc"),
                                          ("mskv_topk_desc", "TopkDesc"), ("mskv_attn_desc", "AttnDesc")])
def test_struct_field_order_matches_header(cname, pyname):
    from mserve_b200 import _lib
    py = [f[0] for f in getattr(_lib, pyname)._fields_]
    assert py == _c_struct_fields(cname)


def test_host_side_errors_without_gpu(built_lib):
    """Argument errors surface as exceptions on the host, before any launch."""
    from mserve_b200 import _lib, cuda_uva
    lib = _lib.lib()
    # NULL descriptors and bad sizes are refused by the C entry points themselves
    assert lib.mskv_gather(None, None) == _lib.MSKV_ERR_ARG
    assert "NULL" in lib.mskv_last_error().decode()
    assert lib.mskv_uva_gather(None, None, None, 1, 1, 1, 1, 1, 2, None, None, None, None) == _lib.MSKV_ERR_ARG
    assert lib.mskv_uva_gather(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 1, 1, 1, 1, 1, 3,
                               C.c_void_p(16), C.c_void_p(16), None, None) == _lib.MSKV_ERR_DTYPE
    d = _lib.TopkDesc()
    d.num_sel, d.rows_per_sel, d.sel_per_batch, d.out_bits = 1, 1, 1, 16
    assert lib.mskv_topk(C.byref(d), None) == _lib.MSKV_ERR_ARG
    # the drop-in refuses pageable host tensors exactly like the reference's TORCH_CHECK
    k = torch.zeros(1, 2, 10, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="pinned"):
        cuda_uva.uva_gather(k, k, torch.tensor([0]), 1, 2, 10, 8)


def test_cpulist_parsing():
    from mserve_b200 import topology
    assert topology.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert topology.parse_cpulist("") == set()


def test_cuda_uva_module_imports_by_name(built_lib):
    """The torch extension answers to the reference's module name and signature, and checks its
    arguments before any GPU work (unpinned host KV raises the reference's error text)."""
    import subprocess
    import sys
    from mserve_b200 import build
    ext = build.build_torch_ext()
    code = ("import sys, torch; sys.path.insert(0, %r); import cuda_uva; "
            "assert cuda_uva.__file__ == %r; "
            "k = torch.zeros(1, 1, 4, 8)\n"
            "try:\n    cuda_uva.uva_gather(k, k, torch.tensor([0]), 1, 1, 4, 8)\n"
            "except RuntimeError as e:\n    print(str(e).splitlines()[0])\n") % (str(ext.parent), str(ext))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "k_in must be pinned memory for UVA" in out.stdout
