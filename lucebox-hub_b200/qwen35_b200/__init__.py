"""B200-native Qwen3.5 hybrid forward path behind lucebox-hub's Decoder API."""
from .config import QWEN35_0P8B, TINY, Dims, MAX_SEQ_LEN  # noqa: F401
