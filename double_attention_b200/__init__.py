"""B200-native (sm_100a) routed-attention hot path of Double Attention."""
