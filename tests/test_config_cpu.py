"""The reference training YAML (keys of chessdecoder/train/config.yaml) maps
onto the fused step's configuration (CPU: the mapping only; the step itself
needs a GPU)."""
import yaml

from chessdecoder_b200.config import load_train_config, model_config

REFERENCE_SHAPED = """
project_name: "chess-decoder"
data: {parquet_dir: "/data/", batch_size: 64, num_workers: 8, max_seq_len: 256, skip_board_prob: 0.2}
model: {embed_dim: 1024, num_heads: 16, num_layers: 12, max_seq_len: 256, d_ff: 1536, n_buckets: 100,
        wl_sigma: 0.4, value_hidden_size: 256, num_fourier_freq: 128}
training: {learning_rate: 1.0e-4, weight_decay: 0.1, gradient_accumulation_steps: 4, num_epochs: 100,
           device: "cuda", use_amp: true, checkpoint_dir: "checkpoints/"}
loss: {move_weight: 5.0, board_weight: 1.0, wl_weight: 1.0, d_weight: 1.0}
"""


def test_model_section_maps_to_model_config(tmp_path):
    p = tmp_path / "config.yaml"
    p.write_text(REFERENCE_SHAPED)
    conf = load_train_config(str(p))
    cfg = model_config(conf)
    assert (cfg.embed_dim, cfg.num_heads, cfg.num_layers, cfg.max_seq_len, cfg.d_ff) == (1024, 16, 12, 256, 1536)
    assert (cfg.n_buckets, cfg.value_hidden_size, cfg.num_fourier_freq, cfg.wl_sigma) == (100, 256, 128, 0.4)
    assert cfg.vocab_size == 1968 and cfg.moe_experts == 0 and not cfg.finetune


def test_kernels_section_selects_variants():
    conf = yaml.safe_load(REFERENCE_SHAPED)
    conf["kernels"] = {"moe_experts": 8, "moe_capacity": 1.5}
    cfg = model_config(conf)
    assert cfg.moe_experts == 8 and cfg.moe_capacity == 1.5
