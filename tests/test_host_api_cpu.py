"""Host-side pieces of the Python drop-in, on CPU tensors: the package's torch
verifier (used by run_quantizer / prepare_and_quantize) and the layout decoder
agree with the CPU oracle, including special values, so the verifier cannot
pass a wrong kernel."""

import numpy as np
import pytest
import torch

import MXFP8_quantizer
import inputs

pkg = MXFP8_quantizer.load_package()


@pytest.mark.parametrize("name,dtype,gen", [
    ("c1", "bf16", lambda: inputs.normal(256, 1024, 0)),
    ("c4", "bf16", lambda: inputs.special_values_bf16()),
    ("nonfinite_bf16", "bf16", lambda: inputs.nonfinite_patterns("bf16")),
    ("nonfinite_fp16", "fp16", lambda: inputs.nonfinite_patterns("fp16")),
    ("sweep_fp16", "fp16", lambda: inputs.amax_sweep("fp16")),
])
def test_torch_verifier_matches_oracle(name, dtype, gen, oracle_mod):
    bits = gen()
    m, k = bits.shape
    km, kk = oracle_mod.padded_shape(m, k)
    x = torch.zeros((km, kk), dtype=torch.bfloat16 if dtype == "bf16" else torch.float16)
    x[:m, :k] = inputs.bits_to_torch(bits, dtype)
    scale, q = pkg.reference_quantize(x)
    q_ref, s_ref = oracle_mod.quantize(bits, dtype, km, kk)
    np.testing.assert_array_equal(q.view(torch.uint8).numpy(), q_ref)
    dense = oracle_mod.unpack_scales(s_ref, km, kk // 32)
    np.testing.assert_array_equal(scale.numpy().astype(np.uint8), dense)


def test_decode_scale_bytes_matches_oracle_layout(oracle_mod):
    bits = inputs.normal(300, 640, 9)
    q, s = oracle_mod.quantize(bits, "bf16", 300, 640)
    dense = pkg.decode_scale_bytes(torch.from_numpy(s), 300, 640).numpy()
    np.testing.assert_array_equal(dense, oracle_mod.unpack_scales(s, 300, 20))


def test_verify_quantizer_outputs_flags_a_wrong_byte(oracle_mod):
    bits = inputs.normal(128, 256, 4)
    q_ref, s_ref = oracle_mod.quantize(bits, "bf16", 128, 256)
    x = inputs.bits_to_torch(bits, "bf16")
    buffers = {"x": x, "q_fp8": torch.from_numpy(q_ref.copy()).view(torch.float8_e4m3fn),
               "s_storage_bytes": torch.from_numpy(s_ref.copy())}
    assert pkg.verify_quantizer_outputs(buffers, 128, 256, 128, 256)["verification_passed"]
    bad = s_ref.copy()
    bad[17] ^= 1
    buffers["s_storage_bytes"] = torch.from_numpy(bad)
    r = pkg.verify_quantizer_outputs(buffers, 128, 256, 128, 256)
    assert not r["scale_bytes_exact"] and not r["verification_passed"]


def test_config_validation_matches_reference_rules():
    with pytest.raises(ValueError):
        pkg.MXFP8QuantizerConfig(torch.bfloat16, rows_per_cta=16).validate()
    with pytest.raises(ValueError):
        pkg.MXFP8QuantizerConfig(torch.bfloat16, k_tile=100).validate()
    with pytest.raises(ValueError):
        pkg.MXFP8QuantizerConfig(torch.float32).validate()
    pkg.MXFP8QuantizerConfig().validate()
    with pytest.raises(ValueError):
        pkg.quantizer._resolve_input_dtype("fp8")
    with pytest.raises(ValueError):
        pkg.run_e2e_verification(m=1000, n=1024, k=2048)        # M not a multiple of the tiler
    with pytest.raises(ValueError):
        pkg.run_e2e_verification(m=1024, n=1024, k=2000)        # K not a multiple of 256
    with pytest.raises(ValueError):
        pkg.run_e2e_verification(mma_tiler_mn=(256, 128), cluster_shape_mn=(1, 1))


def test_quantize_wrapper_rejects_bad_tensors_on_cpu():
    x = torch.zeros((16, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        pkg.quantize(x)                                   # not a CUDA tensor
    with pytest.raises(ValueError):
        pkg.dequantize(torch.zeros((4, 32), dtype=torch.uint8), torch.zeros(512, dtype=torch.uint8))
    with pytest.raises(ValueError):
        pkg.quantize(torch.zeros((2, 3, 4), dtype=torch.bfloat16))
