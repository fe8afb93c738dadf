"""B200-native IndexTTS 2.5 GPT (UnifiedVoice) decode loop.

The product is the shared library built from ``csrc/`` (C-ABI declared in
``include/itts_gpt.h``).  This package also carries its Python binding
(``gpt.py``, ctypes over the C-ABI) and the MIT2 bundle tools (``mit2.py``).
The directory name is not a Python identifier; import it with
``importlib.import_module("index-tts-25-metal_b200")``.
"""
