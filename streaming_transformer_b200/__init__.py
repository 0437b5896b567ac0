"""B200-native streaming-step runtime (package init filled in below)."""
