"""CPU oracle for llmx's attention path (test infrastructure only; see attention.py)."""
from .attention import alibi_slopes, attention_ref, attention_ref_chunked, attention_ref_padded  # noqa: F401
from .merge import merge_partials, merge_row_parts  # noqa: F401
