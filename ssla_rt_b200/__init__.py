"""B200-native SSLA-S per-event hot path (drop-in for haohq19/ssla-rt's
libstage01_to_gpu.so / drain_n path)."""
