"""B200-native (sm_100a) AR-aware 3D block-sparse attention for Light Interaction.

Drop-in modules mirroring the reference's operator surface:

* :mod:`.ar_sparse_operation` — HY-WorldPlay decode (``run_sparse_attention``,
  ``fast_generate_indices``, ``launch_q_prep`` / ``launch_kv_prep`` / ``launch_untile``);
* :mod:`.bi_sparse_operation_for_KV_cache` — HY-WorldPlay prefill
  (``run_sparse_prefill_attention``, ``generate_prefill_indices``);
* :mod:`.bi_sparse_operation` — Matrix-Game-3.0 (``run_sparse_attention``,
  ``generate_prefill_indices``);
* :mod:`.longcat_kernel` — ``longcat_flash_attn``;
* :mod:`.worldplay_acceleration_config` — presets and ``attn_param``;
* :mod:`.memory` — memory-pruning K/V compaction;
* :mod:`.ulysses` — head-sharded multi-GPU step (sequence-to-head all-to-all).

The compute runs in one C-ABI shared library (``_lib/libli_b200.so``,
``include/li_b200.h``) of hand-written CUDA kernels for sm_100a. There is no
CPU or Triton path: without the library or a CUDA device the operators raise.
"""

__version__ = "0.1.0"


def load_native():
    """Load the native library (raises if it has not been built)."""
    from . import _lib
    return _lib.load()


def native_version() -> str:
    return load_native().li_version().decode()
