"""evspark_b200 — B200-native (sm_100a) block-verification hot path for EvSpark."""
