// Exposes the reference's CPU attention loop
// (attention/attention_common.h:123-156) by compiling that header here.
// Test/bench infrastructure only.
#include REF_SOURCE

extern "C" void ref_cpu_attention(const float* q, const float* k,
                                  const float* v, float* out, int batch,
                                  int heads, int seq, int d, int causal) {
  AttentionOptions o;
  o.b = batch;
  o.h = heads;
  o.s = seq;
  o.d = d;
  o.causal = causal != 0;
  AttentionHostData data(o);
  const size_t count = o.tensor_elements();
  std::copy(q, q + count, data.q.begin());
  std::copy(k, k + count, data.k.begin());
  std::copy(v, v + count, data.v.begin());
  std::vector<float> output(count);
  attention_cpu_reference(o, data, output);
  std::copy(output.begin(), output.end(), out);
}
