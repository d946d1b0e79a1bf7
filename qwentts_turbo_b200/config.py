"""Model dimensions of Qwen3-TTS-12Hz-0.6B (talker backbone + code predictor).

Mirrors the constants the reference hard-codes in
``qwentts_turbo/csrc/config.cuh:33-40`` and ``qwentts_turbo/megakernel_backbone.py:14-21``
(backbone) / ``qwentts_turbo/megakernel_code_predictor.py:19-26`` (code predictor).
The CUDA side checks a :class:`ModelDims` against its compiled-in constants at engine
creation (``qtt_engine_create``), so a mismatching checkpoint fails loudly.
"""
from dataclasses import dataclass, field


@dataclass(frozen=True)
class ModelDims:
    hidden: int = 1024
    intermediate: int = 3072
    n_q_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    # mRoPE sections (temporal, height, width) over the 64 rotary frequencies;
    # rope_multimodal.cuh:26-30.
    mrope_section: tuple = (24, 20, 20)
    backbone_layers: int = 28
    cp_layers: int = 5
    vocab: int = 3072            # talker codec vocabulary (codec_embedding / codec_head rows)
    cp_vocab: int = 2048         # rows of each code-predictor embedding table and lm_head
    n_groups: int = 16           # codebooks per 12 Hz frame (group 0 + 15 code-predictor groups)
    # Token id of codec EOS inside the suppressed top-1024 band of the vocabulary.
    # The reference reads it from the checkpoint (generator.py:68); callers with a real
    # checkpoint pass theirs.
    eos_token_id: int = 2150

    @property
    def q_size(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def layer_params(self) -> int:
        h, i = self.hidden, self.intermediate
        linear = h * self.q_size + 2 * h * self.kv_size + self.q_size * h + 3 * h * i
        norms = 2 * h + 2 * self.head_dim
        return linear + norms

    def layer_bytes(self) -> int:
        """bf16 bytes of one decoder layer (31,461,888 B at the 0.6B shape)."""
        return 2 * self.layer_params


DEFAULT_DIMS = ModelDims()


def frame_weight_bytes(d: ModelDims = None, backbone_layers: int | None = None, cp_layers: int | None = None) -> int:
    """Algorithmic weight bytes of one batch-1 frame: backbone layers + final norm + codec head
    once, plus 15 code-predictor passes of (layers + final norm + one lm_head).
    3,309,813,248 B at the 0.6B shape."""
    d = d or DEFAULT_DIMS
    nb = d.backbone_layers if backbone_layers is None else backbone_layers
    nc = d.cp_layers if cp_layers is None else cp_layers
    layer = d.layer_bytes()
    head = 2 * d.vocab * d.hidden
    cp_head = 2 * d.cp_vocab * d.hidden
    return nb * layer + 2 * d.hidden + head + (d.n_groups - 1) * (nc * layer + 2 * d.hidden + cp_head)


def kv_read_bytes_per_frame(position: int, d: ModelDims = None, backbone_layers: int | None = None,
                            cp_layers: int | None = None) -> int:
    """Algorithmic KV bytes of one frame whose backbone step runs at `position`: the backbone
    reads cache rows [0, position] (bf16 K and V, all layers) and writes one row; the code
    predictor's pass 0 touches rows 0-1 and pass g (1..14) reads rows [0, g+1] (132 fp32 row
    reads in total) and the frame writes 16 rows."""
    d = d or DEFAULT_DIMS
    nb = d.backbone_layers if backbone_layers is None else backbone_layers
    nc = d.cp_layers if cp_layers is None else cp_layers
    bb_row = nb * 2 * d.kv_size * 2            # bytes per position, K+V, bf16
    cp_row = nc * 2 * d.kv_size * 4            # fp32
    bb = (position + 1) * bb_row + bb_row      # read [0, position], write position
    cp_reads = 2 + sum(range(3, d.n_groups + 1))   # pass 0 reads 2 rows, pass g reads g+2 rows
    cp = cp_reads * cp_row + d.n_groups * cp_row
    return bb + cp

# Per-layer tensor order of the reference's weight-pointer struct
# (fused_decode_tts.cu:22-34, megakernel_backbone.py:375-387).
LAYER_TENSORS = (
    "input_layernorm",
    "q_proj",
    "k_proj",
    "v_proj",
    "q_norm",
    "k_norm",
    "o_proj",
    "post_attention_layernorm",
    "gate_proj",
    "up_proj",
    "down_proj",
)
