"""B200-native decode hot path of rec (see include/rec_b200.h)."""
