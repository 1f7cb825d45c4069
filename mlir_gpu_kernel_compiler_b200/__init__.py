"""B200-native execution backend for tensorjit's fused kernel plan."""
