// CPU checks of include/cubutterfly/plan.hpp: descriptors, JSON round trip,
// capabilities and the exception contract (no device needed).
#include <cubutterfly/plan.hpp>

#include <cstdio>
#include <string>

int main() {
    int failures = 0;
    auto expect = [&](bool ok, const char* what) {
        if (!ok) {
            std::printf("FAIL %s\n", what);
            ++failures;
        }
    };
    cubutterfly::Transform t;
    t.extents = {5};
    t.batch = 2;
    cubutterfly::Descriptor d(t);
    d.validate();
    expect(d.capabilities_json().find("\"eligible\"") != std::string::npos, "5-point FFT eligible");
    auto copy = cubutterfly::Descriptor::from_json(d.json());
    expect(copy.json() == d.json(), "JSON round trip");
    try {
        cubutterfly::Transform bad = t;
        bad.input_strides = {1, 1};
        cubutterfly::Descriptor x(bad);
        expect(false, "per-axis count check");
    } catch (const std::invalid_argument&) {
    }
    try {
        cubutterfly::Transform fwht;
        fwht.op = CUBUTTERFLY_OPERATOR_FWHT;
        fwht.storage = CUBUTTERFLY_DATA_FP32;
        fwht.extents = {12};  // not a power of two
        cubutterfly::Descriptor x(fwht);
        x.validate();
        expect(false, "invalid descriptor throws");
    } catch (const std::runtime_error& e) {
        expect(std::string(e.what()).find("CUBUTTERFLY_STATUS_INVALID_VALUE") == 0, "status text leads");
    }
    std::printf(failures ? "failed\n" : "ok\n");
    return failures;
}
