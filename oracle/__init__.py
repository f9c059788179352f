"""CPU oracle for llmx's attention path (test infrastructure only; see attention.py)."""
from .attention import alibi_slopes, attention_ref, attention_ref_padded  # noqa: F401
