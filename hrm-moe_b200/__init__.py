"""B200-native routed MoE-FFN forward for HRM-MoE (package stub, filled in below)."""
