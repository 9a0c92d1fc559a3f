"""tread_b200: B200-native (sm_100a) chunk-reuse hot path with tread's engine/store API."""
