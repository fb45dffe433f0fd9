"""CPU tests of the C-ABI boundary: the library loads without a GPU, exports every entry
point include/fletcher_cuda.h declares, and its host-side logic agrees with the weight layout.
No compute calls are made here."""
import ctypes
import os
import re
import subprocess

import pytest

import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fletcher_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(Cuda_[A-Za-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def fl():
    import build
    build.build()
    import fletcher
    return fletcher


def test_header_declares_the_reference_bridge_entry_points():
    # internal/device/cuda_bridge.h:17-53 entry points that the Go wrapper binds
    ref = ["Cuda_Init", "Cuda_GetDeviceCount", "Cuda_SetDevice", "Cuda_FreeContext", "Cuda_Alloc",
           "Cuda_FreeBuffer", "Cuda_CopyToDevice", "Cuda_CopyToHost", "Cuda_GetBufferContents",
           "Cuda_Linear_Fused", "Cuda_LayerNorm", "Cuda_Softmax", "Cuda_Gather", "Cuda_Attention_Fused",
           "Cuda_ApplyRoPE", "Cuda_Synchronize"]
    assert set(ref) <= set(declared_symbols())


def test_library_exports_every_declared_symbol(fl):
    lib = fl.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", fl.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (Cuda_\w+)", out))
    assert exported == set(declared_symbols())


def test_library_is_sm100a_only(fl):
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", fl.LIB_PATH], capture_output=True, text=True).stdout
    archs = set(re.findall(r"sm_\d+a?", out))
    assert archs == {"sm_100a"}, archs


def test_no_gpu_behaviour(fl):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = fl.lib()
    assert lib.Cuda_GetDeviceCount() == 0
    assert not lib.Cuda_Init()
    with pytest.raises(fl.FletcherError):
        fl.Backend()


def test_weight_count_agrees(fl):
    for cfg in (synth.BERT_TINY, synth.NOMIC):
        c = synth.to_c(cfg)
        assert fl.lib().Cuda_Model_WeightCount(ctypes.byref(c)) == synth.weight_count(cfg)


def test_config_struct_layout(fl):
    # FletcherBertConfig: 8 int32 + 2 float = 40 bytes
    assert ctypes.sizeof(synth.CConfig) == 40
