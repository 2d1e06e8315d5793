"""Host arithmetic of bench.py's whole-step roofline (no GPU): the algorithmic units of one
refinement step of the 1.5B model -- weights incl. biases and norms, KV reads over prefix + 32
keys, KV writes of the step's rows -- and the floor time against the HBM and tensor peaks."""

import bench


def test_step_units_match_the_architecture():
    from fast_dllm_relax_b200.config import QWEN_1_5B as c

    per_layer = (c.hidden_size * (c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim  # qkv
                 + c.num_attention_heads * c.head_dim * c.hidden_size                            # o
                 + 3 * c.hidden_size * c.intermediate_size)                                      # gate_up, down
    macs = c.num_hidden_layers * per_layer + c.vocab_size * c.hidden_size
    assert macs == bench.STEP_MACS_PER_ROW
    extra = c.num_hidden_layers * ((c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim  # qkv bias
                                   + 2 * c.hidden_size) + c.hidden_size                            # norms
    assert 2 * (macs + extra) == bench.STEP_WEIGHT_BYTES
    assert bench.KV_BYTES_PER_KEY == c.num_hidden_layers * 2 * c.num_key_value_heads * c.head_dim * 2


def test_step_roofline_is_weight_bound_at_decode_rows():
    r = bench.step_roofline(32, 384, 1.0, 6552.0, 1618.1)
    assert r["bytes"] == 3_087_428_608 + 28_672 * 416 + 28_672 * 32
    m = r["measured"]
    assert abs(m["floor_ms"] - r["bytes"] / 6552e9 * 1e3) < 1e-9  # HBM-bound: bytes, not FLOPs
    assert abs(m["frac"] - m["floor_ms"]) < 1e-12                  # over a 1 ms step
    assert r["nominal"]["floor_ms"] < m["floor_ms"]
    big = bench.step_roofline(8192, 384, 1.0, 6552.0, 1618.1)      # enough rows to turn tensor-bound
    assert abs(big["measured"]["floor_ms"] - big["flops"] / 1618.1e12 * 1e3) < 1e-9


def test_peaks_fall_back_per_key(tmp_path):
    p = tmp_path / "peaks.json"
    assert bench._peak("hbm_gbs", p) == (6650.0, "fallback")  # no file
    p.write_text('{"hbm_gbs": 6552.0}')
    assert bench._peak("hbm_gbs", p) == (6552.0, "measured")
    assert bench._peak("bf16_tflops", p) == (1590.0, "fallback")  # key absent
    p.write_text("not json")
    assert bench._peak("hbm_gbs", p) == (6650.0, "fallback")
    p.write_text('{"hbm_gbs": null, "bf16_tflops": 1618.1}')
    assert bench._peak("hbm_gbs", p) == (6650.0, "fallback")
    assert bench._peak("bf16_tflops", p) == (1618.1, "measured")


def test_projection_bytes_cover_the_step_weights():
    """bench.py's in-situ roofline counts, per projection launch, weights + activations in +
    outputs; over one step's launches the weight part is every matrix once (the step's weight
    bytes less the qkv biases and the norm weights)."""
    from fast_dllm_relax_b200.config import QWEN_1_5B as c
    names = ("qkv", "o", "gate_up", "down")
    w0 = sum(bench._proj_bytes(n, 0) for n in names) * c.num_hidden_layers + bench._proj_bytes("lm_head", 0)
    extra = c.num_hidden_layers * ((c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim
                                   + 2 * c.hidden_size) + c.hidden_size
    assert w0 == bench.STEP_WEIGHT_BYTES - 2 * extra
    # 32 rows: activations in (rows x K) and outputs on top of the weights
    assert bench._proj_bytes("o", 32) - bench._proj_bytes("o", 0) == 32 * c.hidden_size * 2 * 3
