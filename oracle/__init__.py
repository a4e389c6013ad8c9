"""CPU oracle (test infrastructure only): see ``oracle/rel_attn_oracle.py`` (attention) and
``oracle/rel_logits_oracle.py`` (rel_logits producer)."""
from .rel_attn_oracle import (  # noqa: F401
    rel_attn,
    rel_attn_rows,
    round_to_bf16,
    bf16_bits_to_f32,
    f32_to_bf16_bits,
    alignment_offsets,
    rel_attn_torch,
    rel_attn_rows_torch,
    rel_attn_grads_torch,
)
from .rel_logits_oracle import token_positions, log_tau, rel_logits_proj  # noqa: F401
