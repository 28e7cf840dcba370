"""phonon_b200: B200-native Flow-transformer decode step for speech-mac.

The product is the C-ABI library libphonon_cuda.so (include/phonon_cuda.h)
and the C17 drop-in libphonon_transformer_cuda.so that implements speech-mac's
phonon_transformer.h / phonon_q8.h on top of it. This package only builds and
loads them for Python callers (tests, bench).
"""
