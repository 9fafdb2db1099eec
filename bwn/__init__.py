"""bwn: Blackwell-native (sm_100a) inference and fine-tuning for Qwen3.6, DeepSeek V4 Flash
and ESM-2.  Native kernels load from the in-tree extension ``bwn._C`` (``bwn.ops``)."""
__version__ = "0.1.0"
