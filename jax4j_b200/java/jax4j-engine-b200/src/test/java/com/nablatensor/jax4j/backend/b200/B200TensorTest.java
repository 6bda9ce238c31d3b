package com.nablatensor.jax4j.backend.b200;

import static org.junit.jupiter.api.Assertions.assertArrayEquals;
import static org.junit.jupiter.api.Assertions.assertEquals;
import static org.junit.jupiter.api.Assertions.assertInstanceOf;
import static org.junit.jupiter.api.Assertions.assertThrows;
import static org.junit.jupiter.api.Assertions.assertTrue;

import com.nablatensor.jax4j.tensor.BackendRegistry;
import com.nablatensor.jax4j.tensor.ConvSpec;
import com.nablatensor.jax4j.tensor.DType;
import com.nablatensor.jax4j.tensor.Device;
import com.nablatensor.jax4j.tensor.Jit;
import com.nablatensor.jax4j.tensor.QuantType;
import com.nablatensor.jax4j.tensor.Shape;
import com.nablatensor.jax4j.tensor.Tensor;
import com.nablatensor.jax4j.tensor.Tensors;
import com.nablatensor.jax4j.tensor.Transforms;
import com.nablatensor.jax4j.tensor.spi.DeviceBuffer;
import java.lang.foreign.MemorySegment;
import org.junit.jupiter.api.BeforeAll;
import org.junit.jupiter.api.Test;
import org.junit.jupiter.api.condition.EnabledIfSystemProperty;

/**
 * The reference's CudaTensorTest cases (jax4j-engine-cuda CudaTensorTest.java) on the B200
 * backend, plus the QuantizedOps and convolution entry points. Needs a GPU and the native
 * library: {@code -Djax4j.b200.tests=true -Djax4j.b200.lib=/path/to/libjax4j_b200.so}.
 */
@EnabledIfSystemProperty(named = "jax4j.b200.tests", matches = "true")
class B200TensorTest {
  private static final B200Backend BACKEND = new B200Backend();

  @BeforeAll
  static void requireB200() {
    assertTrue(BACKEND.isAvailable(), "a GPU and libjax4j_b200.so are explicitly required");
    assertInstanceOf(B200Backend.class, BackendRegistry.forDevice(Device.cuda()));
  }

  private Tensor array(float[] values, int... dims) {
    return Tensors.arrayOn(values, Shape.of(dims), Device.cuda());
  }

  @Test
  void uploadElementwiseAndReduction() {
    try (Tensor x = array(new float[] {1, 2, 3, 4}, 4);
         Tensor y = x.mul(x).add(3);
         Tensor sum = y.sum()) {
      assertArrayEquals(new float[] {4, 7, 12, 19}, y.toFloatArray(), 1e-5f);
      assertEquals(42, sum.item(), 1e-5f);
    }
  }

  @Test
  void matrixMultiplication() {
    try (Tensor a = array(new float[] {1, 2, 3, 4, 5, 6}, 2, 3);
         Tensor b = array(new float[] {7, 8, 9, 10, 11, 12}, 3, 2);
         Tensor c = a.matmul(b)) {
      assertArrayEquals(new float[] {58, 64, 139, 154}, c.toFloatArray(), 1e-5f);
    }
  }

  @Test
  void deviceFill() {
    try (Tensor x = array(new float[] {1, 2, 3}, 3);
         Tensor filled = x.fullLike(-2.5f)) {
      assertArrayEquals(new float[] {-2.5f, -2.5f, -2.5f}, filled.toFloatArray(), 0f);
    }
  }

  @Test
  void compiledReplayUsesNewInputs() {
    var plan = Jit.compile(x -> x.mul(x).add(3));
    try (Tensor x = array(new float[] {1, 2}, 2);
         Tensor y = array(new float[] {3, 4}, 2);
         Tensor first = plan.apply(x);
         Tensor second = plan.apply(y)) {
      assertArrayEquals(new float[] {4, 7}, first.toFloatArray(), 1e-5f);
      assertArrayEquals(new float[] {12, 19}, second.toFloatArray(), 1e-5f);
      assertEquals(1, plan.cachedPlanCount());
    }
  }

  @Test
  void compiledGradient() {
    try (Tensor x = array(new float[] {1, 2, 3}, 3);
         Tensor grad = Jit.apply(t -> Transforms.grad(v -> v.mul(v).sum(), t), x)) {
      assertArrayEquals(new float[] {2, 4, 6}, grad.toFloatArray(), 1e-5f);
    }
  }

  @Test
  void shapeErrorsAreIllegalArguments() {
    DeviceBuffer a = BACKEND.upload(new float[] {1, 2, 3}, Shape.of(3), DType.F32, Device.cuda());
    DeviceBuffer b = BACKEND.upload(new float[] {1, 2}, Shape.of(2), DType.F32, Device.cuda());
    assertThrows(IllegalArgumentException.class,
        () -> BACKEND.binary(com.nablatensor.jax4j.tensor.Op.ADD, a, b));
    assertThrows(IllegalArgumentException.class, () -> BACKEND.matmul(a, b));
    assertThrows(UnsupportedOperationException.class,
        () -> BACKEND.upload(new float[] {1}, Shape.of(1), DType.F64, Device.cuda()));
    BACKEND.release(a);
    BACKEND.release(a); // idempotent
    BACKEND.release(b);
  }

  /** One Q8_0 block row (fp16 scale + 32 int8): y = d * sum_j q_j x_j, dequantised in the GEMV. */
  @Test
  void quantizedMatvecAndGather() {
    int rows = 2, cols = 32;
    byte[] blob = new byte[rows * 34];
    for (int r = 0; r < rows; r++) {
      blob[r * 34] = 0x00;               // fp16 0.5 = 0x3800, little-endian
      blob[r * 34 + 1] = 0x38;
      for (int j = 0; j < cols; j++) blob[r * 34 + 2 + j] = (byte) ((j - 16) * (r + 1));
    }
    float[] x = new float[cols];
    for (int j = 0; j < cols; j++) x[j] = 0.25f * j;
    assertTrue(BACKEND.supportedQuantTypes().contains(QuantType.Q8_0));
    DeviceBuffer w = BACKEND.uploadQuantized(MemorySegment.ofArray(blob), QuantType.Q8_0,
        Shape.of(rows, cols), Device.cuda());
    DeviceBuffer xv = BACKEND.upload(x, Shape.of(cols), DType.F32, Device.cuda());
    DeviceBuffer add = BACKEND.upload(new float[] {1, -1}, Shape.of(rows), DType.F32, Device.cuda());
    float[] want = new float[rows];
    for (int r = 0; r < rows; r++) {
      double acc = 0;
      for (int j = 0; j < cols; j++) acc += 0.5 * ((j - 16) * (r + 1)) * x[j];
      want[r] = (float) acc;
    }
    assertArrayEquals(want, BACKEND.download(BACKEND.quantMatvec(w, xv)), 1e-3f);
    assertArrayEquals(new float[] {want[0] + 1, want[1] - 1},
        BACKEND.download(BACKEND.quantMatvecAdd(w, xv, add)), 1e-3f);
    float[] row1 = BACKEND.download(BACKEND.quantGatherRow(w, 1));
    for (int j = 0; j < cols; j++) assertEquals(0.5f * ((j - 16) * 2), row1[j], 0f);
    BACKEND.release(w);
  }

  @Test
  void convolutionMatchesDirectLoops() {
    ConvSpec spec = new ConvSpec(2, 5, 5, 3, 3, 1, 1);
    int batch = 2;
    float[] x = new float[batch * spec.inputSize()], w = new float[spec.outChannels() * spec.weightSize()];
    for (int i = 0; i < x.length; i++) x[i] = (float) Math.sin(i);
    for (int i = 0; i < w.length; i++) w[i] = (float) Math.cos(i);
    float[] got;
    try (Tensor xt = array(x, batch, spec.inputSize());
         Tensor wt = array(w, spec.weightShape().dims());
         Tensor y = xt.conv2d(wt, spec)) {
      got = y.toFloatArray();
    }
    int oh = spec.outHeight(), ow = spec.outWidth(), k = spec.kernel(), c = spec.inChannels();
    for (int b = 0; b < batch; b++)
      for (int o = 0; o < spec.outChannels(); o++)
        for (int i = 0; i < oh; i++)
          for (int j = 0; j < ow; j++) {
            double acc = 0;
            for (int ch = 0; ch < c; ch++)
              for (int u = 0; u < k; u++)
                for (int v = 0; v < k; v++) {
                  int yy = i - spec.pad() + u, xx = j - spec.pad() + v;
                  if (yy < 0 || xx < 0 || yy >= spec.inHeight() || xx >= spec.inWidth()) continue;
                  acc += x[b * spec.inputSize() + (ch * spec.inHeight() + yy) * spec.inWidth() + xx]
                      * w[((o * c + ch) * k + u) * k + v];
                }
            assertEquals(acc, got[b * spec.outputSize() + (o * oh + i) * ow + j], 1e-4);
          }
  }
}
