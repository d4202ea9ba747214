"""Constants and enums of the attention path (mlx_primitives/constants.py:16-28, 100-173).

Only the names the attention API uses are kept: the Layout enum, the mask value and the
normalisation epsilon of the reference's online-softmax paths, the reference's head_dim limit
for its kernels, and its dispatch thresholds (kept for API compatibility; the B200 kernels do
not dispatch on sequence length).
"""

from enum import Enum


class Layout(str, Enum):
    """Tensor layout for attention: BSHD = (batch, seq, heads, dim), BHSD = (batch, heads, seq, dim).

    A str enum, so ``layout == "BSHD"`` and ``layout == Layout.BSHD`` both work.
    """

    BSHD = "BSHD"
    BHSD = "BHSD"


# Additive mask value of the reference's CPU/Metal paths (constants.py:100).  The kernels here
# mask with -inf instead; the two differ only for rows with no admissible key at all, which
# the kernels define as O = 0, LSE = -inf.
ATTENTION_MASK_VALUE = -1e38

# head_dim limit of the kernels (the reference's Metal limit is the same, constants.py:104).
METAL_ATTENTION_MAX_HEAD_DIM = 128

# Epsilon the reference adds to the softmax denominator on its tiled/Metal paths
# (constants.py:110).  The B200 kernels normalise by the exact row sum, like MLX SDPA.
METAL_SOFTMAX_EPSILON = 1e-6

# Dispatch thresholds of the reference (constants.py:162-173); unused by the B200 kernels.
FLASH_MAX_SEQ_FOR_REFERENCE = 256
FLASH_SMALL_BATCH_SEQ_THRESHOLD = 512
FLASH_SMALL_BATCH_THRESHOLD = 4
FLASH_MIN_SEQ_FOR_METAL = 64
