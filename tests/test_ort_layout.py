"""CPU: the vendored onnxruntime_c_api.h has ONNX Runtime's binary layout.

ONNX Runtime hands a custom-op library its function table (OrtApi) and reads
the library's op tables (OrtCustomOp) by position, so the library binds to a
real runtime only if every member it uses sits in ORT's slot. A small C
program is compiled against mamba-onnx_b200/csrc/ort/onnxruntime_c_api.h and
prints each member's slot; the test compares them with

* the end slot of each API version's block, the counts ONNX Runtime itself
  asserts for its table (version 1 ends at slot 101 ... version 17 at 275),
* the slot of every OrtApi entry csrc/ort_ops.cc calls, and the member order
  of OrtCustomOp (version 17), OrtApiBase and OrtAllocator.

The same numbers are static_asserts in csrc/ort_ops.cc, so a layout change
also fails the library build.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
ORT_INC = ROOT / "mamba-onnx_b200" / "csrc" / "ort"

VERSION_ENDS = {
    "ReleaseCustomOpDomain": 101, "ReleaseModelMetadata": 118,
    "AddFreeDimensionOverrideByName": 124, "ReleaseAvailableProviders": 126,
    "SetGlobalSpinControl": 149, "ReleaseArenaCfg": 157, "GetCurrentGpuDeviceId": 161,
    "CreateSessionFromArrayWithPrepackedWeightsContainer": 169, "GetSparseTensorIndices": 191,
    "SynchronizeBoundOutputs": 203, "SessionOptionsAppendExecutionProvider_MIGraphX": 209,
    "ReleaseKernelInfo": 218, "ReleaseCANNProviderOptions": 224, "GetSessionConfigEntry": 238,
    "GetBuildInfoString": 254, "KernelContext_GetResource": 265,
    "SessionOptionsAppendExecutionProvider_OpenVINO_V2": 275,
}
USED = {
    "CreateStatus": 0, "GetErrorCode": 1, "GetErrorMessage": 2, "CreateCustomOpDomain": 26,
    "CustomOpDomain_Add": 27, "AddCustomOpDomain": 28, "GetTensorMutableData": 51,
    "GetTensorElementType": 60, "GetDimensionsCount": 61, "GetDimensions": 62,
    "GetTensorTypeAndShape": 65, "KernelContext_GetInputCount": 88,
    "KernelContext_GetOutputCount": 89, "KernelContext_GetInput": 90,
    "KernelContext_GetOutput": 91, "ReleaseStatus": 93, "ReleaseTensorTypeAndShapeInfo": 99,
    "ReleaseAllocator": 132, "KernelContext_GetGPUComputeStream": 193,
    "GetTensorMemoryInfo": 194, "KernelContext_GetAllocator": 253,
}
CUSTOM_OP = ["version", "CreateKernel", "GetName", "GetExecutionProviderType", "GetInputType",
             "GetInputTypeCount", "GetOutputType", "GetOutputTypeCount", "KernelCompute",
             "KernelDestroy", "GetInputCharacteristic", "GetOutputCharacteristic",
             "GetInputMemoryType", "GetVariadicInputMinArity", "GetVariadicInputHomogeneity",
             "GetVariadicOutputMinArity", "GetVariadicOutputHomogeneity", "CreateKernelV2",
             "KernelComputeV2", "InferOutputShapeFn", "GetStartVersion", "GetEndVersion"]


@pytest.fixture(scope="module")
def slots(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    d = tmp_path_factory.mktemp("ort_layout")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "onnxruntime_c_api.h"',
             "int main(void) {"]
    for m in list(VERSION_ENDS) + list(USED):
        lines.append(f'  printf("OrtApi {m} %zu\\n", offsetof(OrtApi, {m}) / sizeof(void*));')
    for m in CUSTOM_OP[1:]:
        lines.append(f'  printf("OrtCustomOp {m} %zu\\n", offsetof(OrtCustomOp, {m}) / '
                     "sizeof(void*));")
    for m in ["GetApi", "GetVersionString"]:
        lines.append(f'  printf("OrtApiBase {m} %zu\\n", offsetof(OrtApiBase, {m}) / '
                     "sizeof(void*));")
    for m in ["Alloc", "Free", "Info"]:
        lines.append(f'  printf("OrtAllocator {m} %zu\\n", offsetof(OrtAllocator, {m}) / '
                     "sizeof(void*));")
    lines.append('  printf("OrtApi sizeof %zu\\n", sizeof(OrtApi) / sizeof(void*));')
    lines += ["  return 0;", "}"]
    src = d / "probe.c"
    src.write_text("\n".join(lines) + "\n")
    exe = d / "probe"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", f"-I{ORT_INC}", str(src), "-o",
                    str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    table = {}
    for line in out.splitlines():
        struct, member, value = line.split()
        table[(struct, member)] = int(value)
    return table


@pytest.mark.parametrize("member", list(VERSION_ENDS))
def test_version_blocks_end_where_ort_ends_them(slots, member):
    assert slots[("OrtApi", member)] == VERSION_ENDS[member]


@pytest.mark.parametrize("member", list(USED))
def test_used_entries_sit_in_ort_slots(slots, member):
    assert slots[("OrtApi", member)] == USED[member]


def test_table_covers_version_17(slots):
    assert slots[("OrtApi", "sizeof")] == 276


def test_custom_op_member_order(slots):
    # OrtCustomOp starts with a uint32_t version, padded to a pointer
    for i, m in enumerate(CUSTOM_OP[1:], start=1):
        assert slots[("OrtCustomOp", m)] == i, m


def test_api_base_and_allocator(slots):
    assert slots[("OrtApiBase", "GetApi")] == 0 and slots[("OrtApiBase", "GetVersionString")] == 1
    assert [slots[("OrtAllocator", m)] for m in ["Alloc", "Free", "Info"]] == [1, 2, 3]
