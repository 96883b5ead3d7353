"""B200-native torch.compile backend (drop-in for the reference's `compiler`
package: compiler.backend.custom_backend, compiler.optimization.*)."""
