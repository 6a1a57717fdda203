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


@pytest.mark.skipif(not os.path.isdir(REFERENCE_INCLUDE), reason="reference headers not present here")
def test_cpp_backend_compiles_with_reference_tensor(tmp_path):
    # the wrapper instantiates with the reference's own infvino::Tensor type
    compile_driver(str(tmp_path), ["-DWITH_REFERENCE_TENSOR", "-I" + REFERENCE_INCLUDE])


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
