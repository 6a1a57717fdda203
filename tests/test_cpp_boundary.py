"""The C++ drop-in (include/infvino_b200_backend.hpp) compiles against the C ABI
and behaves like ClBackend; on a GPU it reproduces the Python path's outputs."""
import os
import subprocess

import numpy as np
import pytest

import infvino_b200 as ivb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE_INCLUDE = os.path.join(os.environ.get("INFVINO_REFERENCE", "/root/reference"), "include")


def compile_driver(tmp, extra=()):
    exe = os.path.join(tmp, "backend_driver")
    lib = os.path.dirname(ivb._native.LIB_PATH)
    ivb.lib()  # make sure the library is built
    cmd = ["g++", "-std=c++17", "-O1", os.path.join(ROOT, "tests", "cpp", "backend_driver.cpp"),
           "-I" + os.path.join(ROOT, "include"), *extra, "-L" + lib, "-linfvino_b200",
           "-Wl,-rpath," + lib, "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_backend_compiles_and_reports_empty_plan(tmp_path):
    exe = compile_driver(str(tmp_path))
    r = subprocess.run([exe, "--empty-plan"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ModelInfo.plan is empty" in r.stdout


REFERENCE_TYPES = ["-DWITH_REFERENCE_TYPES", "-I" + REFERENCE_INCLUDE,
                   "-I" + os.path.join(ROOT, "oracle", "cvshim"), "-I" + os.path.join(ROOT, "tests", "cpp", "refshim")]


@pytest.mark.skipif(not os.path.isdir(REFERENCE_INCLUDE), reason="reference headers not present here")
def test_cpp_backend_compiles_with_reference_types(tmp_path):
    """The drop-in instantiates with the reference's own infvino::Tensor,
    infvino::ModelInfo and infvino::DeviceInfo (device() returns the caller's
    DeviceInfo, so InferenceEngine::device() forwards it unchanged), and
    reports the reference's empty-plan error."""
    exe = compile_driver(str(tmp_path), REFERENCE_TYPES)
    r = subprocess.run([exe, "--empty-plan"], capture_output=True, text=True)
    assert r.returncode == 0 and "ModelInfo.plan is empty" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_cpp_backend_matches_python_path(tmp_path, model_plans):
    exe = compile_driver(str(tmp_path))
    plan = model_plans["mobilenetv3-small"]
    n = 3 * 224 * 224
    a = np.random.default_rng(1).random(n, dtype=np.float32)
    b = np.random.default_rng(2).random(n, dtype=np.float32)
    a.tofile(tmp_path / "a.f32")
    b.tofile(tmp_path / "b.f32")
    r = subprocess.run([exe, plan, str(tmp_path / "a.f32"), str(tmp_path / "b.f32"), str(tmp_path / "o.f32")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(tmp_path / "o.f32", dtype=np.float32)
    m = ivb.PlanModel(plan)
    ref = m.infer_f32(b, 1)[0]
    assert np.array_equal(got, ref)


@pytest.mark.gpu
def test_cpp_backend_decode_pose_matches_python_path(tmp_path, plan_dir):
    """decodePose() of the C++ drop-in returns the detections of the Python
    path's decodePose (both over ivc_decode_pose) for the same image."""
    from infvino_b200 import plangen
    exe = compile_driver(str(tmp_path))
    plan = plangen.yolov8n_pose(os.path.join(plan_dir, "y8_peaked_cpp"), cls_gain=100.0, cls_shift=-3.0)
    x = np.random.default_rng(7).random(3 * 640 * 640, dtype=np.float32)
    x.tofile(tmp_path / "x.f32")
    r = subprocess.run([exe, "--pose", plan, str(tmp_path / "x.f32"), str(tmp_path / "d.f32")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(tmp_path / "d.f32", dtype=np.float32).reshape(-1, 6 + 34)
    m = ivb.PlanModel(plan)
    m.infer_f32(x, 1)
    ref = m.decodePose(1)[0]
    assert got.shape[0] > 0 and np.array_equal(got, ref)


@pytest.mark.gpu
def test_cpp_plan_model_drives_like_the_tools(tmp_path, model_plans):
    """The C++ PlanModel (setInput once, run twice under profiling, readOutput,
    readTensor, profile(), pool statistics) gives the Python path's output."""
    exe = compile_driver(str(tmp_path))
    plan = model_plans["mobilenetv3-small"]
    x = np.random.default_rng(4).random(3 * 224 * 224, dtype=np.float32)
    x.tofile(tmp_path / "x.f32")
    r = subprocess.run([exe, "--planmodel", plan, str(tmp_path / "x.f32"), str(tmp_path / "y.f16")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(tmp_path / "y.f16", dtype=np.uint16)
    m = ivb.PlanModel(plan)
    m.setInput(ivb.f32_to_f16(x), 1)
    m.run(1)
    assert np.array_equal(got, m.readOutput(0, 1))


@pytest.mark.gpu
def test_cpp_device_info(tmp_path, model_plans):
    """device() fills the DeviceInfo fields from the CUDA device, with the
    reference's own DeviceInfo type when its headers are present."""
    extra = REFERENCE_TYPES if os.path.isdir(REFERENCE_INCLUDE) else []
    exe = compile_driver(str(tmp_path), extra)
    r = subprocess.run([exe, "--device", model_plans["mobilenetv3-small"]], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "CUDA:0" in r.stdout
