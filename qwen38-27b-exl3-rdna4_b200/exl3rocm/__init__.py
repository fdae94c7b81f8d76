"""exl3rocm: the EXL3 inference hot path on NVIDIA B200 (sm_100a), drop-in for the reference's
vLLM plugin package of the same name (Luke458/qwen38-27b-exl3-rdna4, vllm_plugin/exl3rocm).

Importing the package does not import vLLM; ``exl3rocm.plugin.register`` (the
``vllm.general_plugins`` entry point) does.  Every op runs on libexl3b.so; there is no CPU path.
"""
__version__ = "0.1.0"
