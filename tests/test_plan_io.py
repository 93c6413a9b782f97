"""Host-side tests of the plan format (no GPU): the ONNX writer in
inferc_b200.onnx_io against the library's C++ wire-format reader
(inferc_dev_graph_describe parses without touching a device), and the
synthetic optimized plans' op inventory (the fusion counts the reference's
correctness test expects for DistilBERT, tests/correctness_test.cc:134-144:
6 FusedQKV / 6 FusedAttention / 13 FusedLayerNorm / 6 FusedMatMulAddGELU)."""
import numpy as np
import pytest

from inferc_b200 import executor, lib, onnx_io, plan_synth, synth


def test_writer_reader_round_trip_of_every_field_kind():
    g = onnx_io.GraphBuilder("probe")
    g.input("x", onnx_io.FLOAT, ["batch", 4])
    g.init("w", np.arange(12, dtype=np.float32).reshape(3, 4))
    g.init("ids", np.array([-1, 2, 300000], np.int64))
    g.init("flag", np.array([True, False]))
    g.add("Gemm", ["x", "w"], outputs=["y"], transB=1, alpha=0.5)
    g.add("Constant", [], outputs=["c"], value=np.array([1.5], np.float32))
    g.add("Transpose", ["y"], outputs=["t"], perm=[1, 0])
    g.add("FusedAttention", ["t", "t", "t"], outputs=["o"], domain="inferc", head_dim=64,
          fill=-3.0e38)
    g.output("o", onnx_io.FLOAT, ["batch", 3])
    d = executor.describe(g.model())
    assert d["nodes"] == 4 and d["initializers"] == 3
    assert d["initializer_elements"] == 12 + 3 + 2
    assert d["ops"] == {"Gemm": 1, "Constant": 1, "Transpose": 1, "inferc:FusedAttention": 1}
    assert ["inferc", 1] in d["opsets"] and ["", 17] in d["opsets"]
    assert d["inputs"] == [{"name": "x", "dtype": 1, "shape": [-1, 4]}]
    assert d["outputs"] == [{"name": "o", "dtype": 1, "shape": [-1, 3]}]


def test_malformed_bytes_are_rejected_with_a_message():
    L = lib.load()
    good = onnx_io.GraphBuilder("g").model()
    for bad in (good[:-3], b"\x3a\xff\xff\xff\xff\x0f", b"\x0b"):
        rc = L.inferc_dev_graph_describe(bad, len(bad), None, 0, None)
        assert rc == 1
        assert b"ONNX parse error" in L.inferc_dev_last_error_string()


def test_unsupported_op_is_rejected_at_load_before_any_device_work():
    g = onnx_io.GraphBuilder("g")
    g.add("LSTM", ["x"], outputs=["y"])
    m = g.model()
    import ctypes
    h = ctypes.c_void_p()
    L = lib.load()
    rc = L.inferc_dev_graph_load(m, len(m), ctypes.byref(h))
    assert rc == 1
    assert b"unsupported op 'LSTM'" in L.inferc_dev_last_error_string()


def test_distilbert_plan_inventory():
    cfg = synth.EncoderConfig(layers=6, hidden=64, heads=4, ffn=128, vocab=500, max_pos=64)
    d = executor.describe(plan_synth.distilbert_plan(cfg, synth.encoder_weights(cfg, seed=0)))
    ops = d["ops"]
    assert ops["inferc:FusedQKV"] == 6 and ops["inferc:FusedAttention"] == 6
    assert ops["inferc:FusedLayerNorm"] == 13 and ops["inferc:FusedMatMulAddGELU"] == 6
    assert ops["Gemm"] == 2 and ops["Relu"] == 1 and ops["Equal"] == 1
    assert [i["name"] for i in d["inputs"]] == ["input_ids", "attention_mask"]
    assert d["outputs"] == [{"name": "logits", "dtype": 1, "shape": [-1, 2]}]


@pytest.mark.parametrize("with_past", [False, True])
def test_gpt2_plans_inventory(with_past):
    cfg = synth.Gpt2Config(layers=2, hidden=64, heads=4, ffn=256, vocab=300, max_pos=64)
    a, b = plan_synth.gpt2_plans(cfg, synth.gpt2_weights(cfg, seed=0))
    d = executor.describe(b if with_past else a)
    names = [i["name"] for i in d["inputs"]]
    assert names[:2] == ["input_ids", "attention_mask"]
    assert (len(names) == 2 + 2 * cfg.layers) == with_past
    outs = [o["name"] for o in d["outputs"]]
    assert outs[0] == "logits" and "present.1.value" in outs
    assert d["ops"]["inferc:GeluTanh"] == cfg.layers
    assert d["ops"]["inferc:FusedLayerNorm"] == 2 * cfg.layers + 1
    assert d["ops"]["Softmax"] == cfg.layers and d["ops"]["Where"] == cfg.layers
    assert d["ops"].get("Concat", 0) == (2 * cfg.layers + 2 if with_past else 2)


def test_scalar_initializer_has_no_dims():
    # TensorProto of a 0-d array: data_type, name and raw_data only (no dims
    # field), so the reader sees rank 0
    t = onnx_io.tensor("c", np.asarray(1, np.int64))
    assert t == bytes.fromhex("1007") + bytes.fromhex("4201") + b"c" + bytes.fromhex(
        "4a080100000000000000")
