package com.nablatensor.jax4j.backend.b200;

/** AadEngine "cuda-eager": one launch per tape node over scenario slots; engine option "bytes" (scratch budget). */
public final class B200EagerEngine extends B200AadEngines.Base {
  public B200EagerEngine() {
    super("cuda-eager", 81, B200AadEngines.EAGER, "bytes");
  }
}
