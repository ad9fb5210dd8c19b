"""The C++ layer of libnq, driven through tests/cpp/backend_check.cpp: the
CUDABackend lifecycle (mlx_backend.cpp:30-50), cuda_ops::bits (mlx_ops.h:20-25),
config.json's quantization block (model_config.cpp:177-193), the safetensors
reader and loader (model_loader.cpp:17-58) and cuda_ops::lin over a loaded
checkpoint (mlx_ops.h:28-42), the last one against the oracle on a GPU."""
import json
import os
import struct
import subprocess

import numpy as np
import pytest

from _util import acts, assert_close, weights

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def checker(nqlib, tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("cpp") / "backend_check")
    lib_dir = os.path.join(ROOT, "neurons_b200")
    subprocess.run(["g++", "-std=c++23", "-O1", "-I" + os.path.join(lib_dir, "csrc"),
                    "-I" + os.path.join(lib_dir, "csrc", "iface"),
                    "-I" + os.path.join(ROOT, "include"), "-I/usr/local/cuda/include",
                    os.path.join(ROOT, "tests", "cpp", "backend_check.cpp"), "-o", exe,
                    "-L" + lib_dir, "-lnq", "-L/usr/local/cuda/lib64", "-lcudart",
                    "-Wl,-rpath," + lib_dir], check=True)

    def run(*args):
        out = subprocess.run([exe] + [str(a) for a in args], capture_output=True, text=True,
                             timeout=300)
        assert out.returncode == 0, out.stderr
        return [line.split() for line in out.stdout.splitlines()]
    return run


def write_safetensors(path, tensors, metadata=None):
    """tensors: name -> (dtype string, numpy array), written in insertion order."""
    header, blobs, off = {}, [], 0
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = metadata or {"format": "mlx"}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def test_backend_lifecycle(checker):
    import torch
    out = dict((r[0], r[1:]) for r in checker("backend"))
    assert out["type_cuda"] == ["1"]
    if torch.cuda.is_available():
        assert out["available"] == ["1"] and out["initialize"] == ["ok"]
        assert out["stream"] == ["1"] and out["synchronize"] == ["ok"] and out["cleanup"] == ["ok"]
    else:
        assert out["available"] == ["0"] and out["initialize"] == ["BackendNotAvailable"]


def test_bits_like_mlx_ops(checker, oracle):
    got = [int(r[1]) for r in checker("bits")]
    want = [oracle.bits_from_shapes(w, s, g) for w, s, g in ((512, 64, 64), (1024, 64, 64),
                                                             (96, 12, 64), (0, 64, 64))]
    assert got == want == [4, 8, 4, 4]


@pytest.mark.parametrize("cfg,expect", [
    ({"model_type": "llama", "quantization": {"group_size": 64, "bits": 4}}, ["64", "4"]),
    ({"model_type": "llama", "quantization": {"bits": 8, "group_size": 32, "mode": "affine"}},
     ["32", "8"]),
    ({"model_type": "llama"}, ["none"]),
    ({"model_type": "llama", "quantization": None}, ["none"]),
])
def test_quantization_config(checker, tmp_path, cfg, expect):
    (tmp_path / "config.json").write_text(json.dumps(cfg, indent=2))
    out = checker("config", tmp_path)
    assert out[0][0] == "quantization" and out[0][1:] == expect


@pytest.mark.parametrize("text", ['{"quantization": {"bits": 4}}',
                                  '{"quantization": {"group_size": 64}}',
                                  '{"quantization": {"group_size": 64, "bits": 4}',
                                  'not json'])
def test_quantization_config_rejects(checker, tmp_path, text):
    (tmp_path / "config.json").write_text(text)
    assert checker("config", tmp_path)[0] == ["error", "InvalidInput"]


def test_safetensors_header(checker, tmp_path):
    f = tmp_path / "model.safetensors"
    write_safetensors(f, {
        "model.layers.0.mlp.up_proj.weight": ("U32", np.arange(24, dtype=np.uint32).reshape(3, 8)),
        "model.layers.0.mlp.up_proj.scales": ("BF16", np.zeros((3, 1), np.uint16)),
        "model.embed_tokens.scales": ("F16", np.zeros((5, 2), np.uint16)),
        "model.norm.weight": ("F32", np.ones(7, np.float32)),
    }, metadata={"format": "mlx", "note": "café \"quoted\""})
    out = checker("header", f)
    assert out[0][0] == "data_offset" and int(out[0][1]) % 8 == 0
    tensors = {r[1]: (r[2], [int(v) for v in r[3:]]) for r in out[1:]}
    assert tensors == {"model.layers.0.mlp.up_proj.weight": ("U32", [3, 8]),
                       "model.layers.0.mlp.up_proj.scales": ("BF16", [3, 1]),
                       "model.embed_tokens.scales": ("F16", [5, 2]),
                       "model.norm.weight": ("F32", [7])}


def test_safetensors_header_rejects(checker, tmp_path):
    bad = tmp_path / "bad.safetensors"
    # data range does not match the shape
    h = json.dumps({"w": {"dtype": "U32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 16)
    assert checker("header", bad)[0] == ["error", "InvalidInput"]
    # unsupported dtype
    h = json.dumps({"w": {"dtype": "F64", "shape": [2], "data_offsets": [0, 16]}}).encode()
    bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 16)
    assert checker("header", bad)[0] == ["error", "InvalidInput"]
    # header length past the end of the file
    bad.write_bytes(struct.pack("<Q", 1 << 20) + b"{}")
    assert checker("header", bad)[0] == ["error", "InvalidInput"]


@pytest.mark.gpu
@pytest.mark.parametrize("bits,gs", [(4, 64), (8, 32)])
def test_lin_over_loaded_checkpoint(checker, oracle, tmp_path, bits, gs):
    """Two files (sorted, merged like load_model_mlx), quantized in MLX's layout;
    cuda_ops::lin on the loaded map against the oracle."""
    rng = np.random.default_rng(bits)
    N, K, M = 192, 512, 5
    wq, s, b = oracle.quantize(weights(rng, N, K), bits, gs, 0)
    key = "model.layers.0.mlp.up_proj"
    write_safetensors(tmp_path / "model-00001-of-00002.safetensors",
                      {key + ".weight": ("U32", wq), key + ".scales": ("BF16", s)})
    write_safetensors(tmp_path / "model-00002-of-00002.safetensors",
                      {key + ".biases": ("BF16", b),
                       "model.norm.weight": ("BF16", np.zeros(K, np.uint16))})
    (tmp_path / "config.json").write_text(json.dumps(
        {"model_type": "llama", "quantization": {"group_size": gs, "bits": bits}}))
    x = acts(rng, M, K)
    x.tofile(tmp_path / "x.bin")
    out = checker("lin", tmp_path, key, tmp_path / "x.bin", M, K, tmp_path / "y.bin")
    assert out[0][0] == "tensors" and int(out[0][1]) == 4, out
    assert out[-1][:2] == ["lin", "ok"], out
    y = np.fromfile(tmp_path / "y.bin", np.uint16).reshape(M, N)
    assert_close(y, oracle.qmm(x, wq, s, b, bits, gs), f"lin {bits}-bit g{gs}")


@pytest.mark.gpu
def test_lin_dense_weight_falls_back_to_matmul(checker, oracle, tmp_path):
    """A layer stored without scales (an unquantized projection) goes through
    mlx_ops::lin's plain matmul branch (mlx_ops.h:40): y = x . W^T, bf16 in,
    fp32 accumulation, bf16 out."""
    rng = np.random.default_rng(11)
    N, K, M = 96, 256, 5
    w = oracle.f32_to_bf16(weights(rng, N, K))
    key = "lm_head"
    write_safetensors(tmp_path / "model.safetensors", {key + ".weight": ("BF16", w)})
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "llama"}))
    x = acts(rng, M, K)
    x.tofile(tmp_path / "x.bin")
    out = checker("lin", tmp_path, key, tmp_path / "x.bin", M, K, tmp_path / "y.bin")
    assert out[-1][:2] == ["lin", "ok"], out
    y = np.fromfile(tmp_path / "y.bin", np.uint16).reshape(M, N)
    ref = oracle.bf16_to_f32(x).astype(np.float64) @ oracle.bf16_to_f32(w).astype(np.float64).T
    assert_close(y, oracle.f32_to_bf16(ref.astype(np.float32)), "dense lin")


@pytest.mark.gpu
def test_lin_over_f16_checkpoint(checker, oracle, tmp_path):
    """A checkpoint whose scales and biases are F16 goes through cuda_ops::lin
    with fp16 activations (M=5: the tcgen05 path; the C++ checker passes x in
    the scales' dtype)."""
    from test_gpu_f16 import assert_close_f16, f16_bits
    rng = np.random.default_rng(21)
    N, K, M, bits, gs = 192, 1024, 5, 4, 64
    wq, s, b = oracle.quantize(f16_bits(weights(rng, N, K)), bits, gs, 0, f16=True)
    key = "model.layers.0.self_attn.o_proj"
    write_safetensors(tmp_path / "model.safetensors",
                      {key + ".weight": ("U32", wq), key + ".scales": ("F16", s),
                       key + ".biases": ("F16", b)})
    (tmp_path / "config.json").write_text(json.dumps(
        {"model_type": "llama", "quantization": {"group_size": gs, "bits": bits}}))
    x = f16_bits(rng.standard_normal((M, K)))
    x.tofile(tmp_path / "x.bin")
    out = checker("lin", tmp_path, key, tmp_path / "x.bin", M, K, tmp_path / "y.bin")
    assert out[-1][:2] == ["lin", "ok"], out
    y = np.fromfile(tmp_path / "y.bin", np.uint16).reshape(M, N)
    assert_close_f16(y, oracle.qmm(x, wq, s, b, bits, gs, f16=True), "fp16 checkpoint lin")
