"""kinetic_rt -- B200-native decoder hot path behind Kinetic-RT's API."""
