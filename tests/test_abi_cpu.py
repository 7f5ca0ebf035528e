"""CPU: the C-ABI library loads and exports every symbol include/*.h declares,
and the generated codebook tables equal the reference's and gguf-py's."""
import ctypes
import re

import numpy as np
import pytest

from sepia_b200 import lib as L

REF_ABI = ["sepia_gpu_available", "sepia_gpu_init", "sepia_gpu_shutdown", "sepia_gpu_device_name",
           "sepia_gpu_wrap_mmap", "sepia_gpu_alloc", "sepia_gpu_free", "sepia_gpu_host_ptr", "sepia_gpu_gpu_addr",
           "sepia_gpu_selftest_touch", "sepia_gpu_begin", "sepia_gpu_flush", "sepia_gpu_end", "sepia_gpu_rmsnorm",
           "sepia_gpu_matvec", "sepia_gpu_silu_mul", "sepia_gpu_add", "sepia_gpu_softmax", "sepia_gpu_sconv",
           "sepia_gpu_matvec_q", "sepia_gpu_dequant_rows", "sepia_gpu_rel_project", "sepia_gpu_banded_attn",
           "sepia_gpu_matvec_off", "sepia_gpu_rmsnorm_off", "sepia_gpu_sconv_off", "sepia_gpu_rel_project_off",
           "sepia_gpu_copy", "sepia_gpu_scale", "sepia_gpu_sconv_hist_roll"]


def test_header_declares_reference_abi():
    names = L.header_symbols()
    assert len(REF_ABI) == 30
    for n in REF_ABI:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = L.load()          # loads without a GPU (no compute calls)
    for n in L.header_symbols():
        assert hasattr(lib, n), n
        assert n in L._PROTOS, f"{n} missing a ctypes prototype"


def test_matches_reference_header(reference_dir):
    """Every function of the reference's src/sepia_gpu.h is declared here with
    the same parameter list (modulo whitespace and parameter names)."""
    def decls(text):
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        out = {}
        for m in re.finditer(r"([A-Za-z_][\w \*]*?)\b(sepia_gpu_\w+)\s*\(([^)]*)\)\s*;", text):
            args = [re.sub(r"\s+", " ", a.strip()) for a in m.group(3).split(",")]
            types = [re.sub(r"\b\w+$", "", a).replace(" ", "") if a != "void" else "void" for a in args]
            out[m.group(2)] = (m.group(1).replace(" ", ""), types)
        return out
    ref = decls((reference_dir / "src" / "sepia_gpu.h").read_text())
    mine = decls((L.INCLUDE / "sepia_gpu.h").read_text())
    assert set(ref) <= set(mine)
    for k, v in ref.items():
        assert mine[k] == v, k


def test_quant_tables_match_reference(reference_dir):
    ours = (L.HERE / "csrc" / "quant_tables.h").read_text()
    theirs = (reference_dir / "src" / "quants_grids.h").read_text()

    def table(text, name):
        m = re.search(name + r"\[\d+\]\s*=\s*\{(.*?)\};", text, re.S)
        vals = re.findall(r"-?0x[0-9a-fA-F]+|-?\d+", m.group(1))
        return [int(v.rstrip("uUlL"), 0) for v in vals]
    for mine, ref in [("sepia_iq2xs_grid", "iq2xs_grid"), ("sepia_iq3xxs_grid", "iq3xxs_grid"),
                      ("sepia_ksigns_iq2xs", "ksigns_iq2xs"), ("sepia_kmask_iq2xs", "kmask_iq2xs"),
                      ("sepia_kvalues_iq4nl", "kvalues_iq4nl")]:
        assert table(ours, mine) == table(theirs, ref), mine


def test_quant_tables_match_gguf():
    from gguf import quants as gq
    ours = (L.HERE / "csrc" / "quant_tables.h").read_text()
    for name, cls in [("sepia_iq2xxs_grid", gq.IQ2_XXS), ("sepia_iq1s_grid", gq.IQ1_S)]:
        m = re.search(name + r"\[\d+\]\s*=\s*\{(.*?)\};", ours, re.S)
        vals = [int(v.rstrip("uUlL"), 0) for v in re.findall(r"0x[0-9a-fA-F]+", m.group(1))]
        cls.init_grid()
        g = np.asarray(cls.grid).reshape(cls.grid_shape).astype(np.int64)
        packed = [sum((int(b) & 0xFF) << (8 * j) for j, b in enumerate(r)) for r in g]
        assert vals == packed, name
